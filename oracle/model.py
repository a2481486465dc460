"""ORACLE (test infrastructure only): torchtune-free fp32 restatement of ChessDecoder.

Used by tests/, ``__graft_entry__.smoke()`` and bench.py's CPU baseline as the
checker / CPU reference.  Never imported by the product package.

Follows chessdecoder/models/model.py:
  * constructor :75-136, in the same parameter-construction order (embedding;
    per layer q, k, v, output projections, then gate (w1), down (w2), up (w3)
    as FeedForward's keyword arguments are evaluated; heads; value heads;
    Fourier frequencies then projection) so ``torch.manual_seed`` gives the
    reference's initial weights; state-dict keys use torchtune's names
    (layers.i.attn.{q,k,v,output}_proj, layers.i.mlp.w1/w2/w3,
    layers.i.{sa,mlp}_norm.scale, norm.scale);
  * forward :138-187 (mask :160-171, embedding + Fourier override :174-180);
  * layer math as restated by the reference at
    chessdecoder/export/backbone_causal.py:108-150 (pre-norm RMSNorm eps 1e-6 in
    fp32, interleaved RoPE from a [max_seq_len, hd/2, 2] cache, SDPA with
    scale 1/sqrt(hd), SwiGLU, residual adds);
  * RoPE cache: torchtune 0.6.1 ``RotaryPositionalEmbeddings`` (third-party,
    absent here) as published: theta_i = base^(-2i/dim), base = 10000,
    cache[p, i] = (cos(p*theta_i), sin(p*theta_i)).  The cache VALUES are not
    pinned by any reference test or fixture (torchtune is not importable here);
    everything downstream of the cache is pinned by tests/golden.
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F

BOARD_VOCAB_SIZE = 41   # chessdecoder/models/vocab.py:245-252 (pinned by tests/test_vocab.py)
MOVE_VOCAB_SIZE = 1924  # chessdecoder/models/vocab.py:255-258
VOCAB_SIZE = 1968


def make_wl_buckets(n_buckets=100, sigma=0.4):
    """model.py:12-16 — Gaussian-quantile WL bucket centres clamped to [-1, 1]."""
    t = torch.linspace(0.5 / n_buckets, 1 - 0.5 / n_buckets, n_buckets)
    return (sigma * math.sqrt(2) * torch.erfinv(2 * t - 1)).clamp(-1.0, 1.0)


def make_d_buckets(n_buckets=100):
    """model.py:19-21 — uniform D bucket centres in [0, 1]."""
    return torch.linspace(0.5 / n_buckets, 1 - 0.5 / n_buckets, n_buckets)


def rope_cache(max_seq_len: int, dim: int, base: float = 10000.0) -> torch.Tensor:
    theta = 1.0 / (base ** (torch.arange(0, dim, 2)[: dim // 2].float() / dim))
    idx = torch.arange(max_seq_len, dtype=theta.dtype)
    ang = torch.einsum("i,j->ij", idx, theta).float()
    return torch.stack([torch.cos(ang), torch.sin(ang)], dim=-1)


class RMSNorm(nn.Module):
    def __init__(self, dim, eps=1e-6):
        super().__init__()
        self.eps = eps
        self.scale = nn.Parameter(torch.ones(dim))

    def forward(self, x):
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps)).type_as(x) * self.scale


class Attention(nn.Module):
    def __init__(self, q, k, v, o, num_heads, head_dim):
        super().__init__()
        self.q_proj, self.k_proj, self.v_proj, self.output_proj = q, k, v, o
        self.num_heads, self.head_dim = num_heads, head_dim


class FeedForward(nn.Module):
    def __init__(self, gate, down, up):
        super().__init__()
        self.w1, self.w2, self.w3 = gate, down, up

    def forward(self, x):
        return self.w2(F.silu(self.w1(x)) * self.w3(x))


class Layer(nn.Module):
    def __init__(self, attn, mlp, sa_norm, mlp_norm):
        super().__init__()
        self.attn, self.mlp, self.sa_norm, self.mlp_norm = attn, mlp, sa_norm, mlp_norm


def apply_rope(x, cache, input_pos):
    """x [B, S, H, hd]; interleaved pairs (backbone_causal.py:66-75)."""
    rv = cache[input_pos].unsqueeze(2)  # [B|1, S, 1, hd/2, 2]
    xs = x.float().reshape(*x.shape[:-1], -1, 2)
    out = torch.stack([xs[..., 0] * rv[..., 0] - xs[..., 1] * rv[..., 1],
                       xs[..., 1] * rv[..., 0] + xs[..., 0] * rv[..., 1]], dim=-1)
    return out.flatten(3).type_as(x)


class FourierEncoder(nn.Module):
    """model.py:24-36."""

    def __init__(self, embed_dim, num_frequencies=128):
        super().__init__()
        self.frequencies = nn.Parameter(torch.randn(1, num_frequencies))
        self.proj = nn.Linear(2 * num_frequencies, embed_dim)

    def forward(self, x):
        f = 2 * math.pi * x.unsqueeze(-1) @ self.frequencies
        return self.proj(torch.cat([f.cos(), f.sin()], dim=-1))


class ValueHead(nn.Module):
    """model.py:39-52."""

    def __init__(self, embed_dim, n_buckets=100, hidden_size=256):
        super().__init__()
        self.mlp = nn.Sequential(nn.Linear(embed_dim, hidden_size), nn.Mish(), nn.Linear(hidden_size, n_buckets))

    def forward(self, h):
        return self.mlp(h)


class OracleChessDecoder(nn.Module):
    def __init__(self, vocab_size, embed_dim=768, num_heads=12, num_layers=12, max_seq_len=2048, d_ff=None,
                 n_buckets=100, value_hidden_size=256, num_fourier_freq=128, wl_sigma=0.4, moe_experts=0,
                 moe_capacity=1.25):
        super().__init__()
        head_dim = embed_dim // num_heads
        d_ff = d_ff if d_ff is not None else 4 * embed_dim
        self.num_heads, self.head_dim = num_heads, head_dim
        self.tok_embedding = nn.Embedding(vocab_size, embed_dim)
        self.register_buffer("rope", rope_cache(max_seq_len, head_dim), persistent=False)
        self.layers = nn.ModuleList()
        for _ in range(num_layers):
            q = nn.Linear(embed_dim, embed_dim, bias=False)
            k = nn.Linear(embed_dim, embed_dim, bias=False)
            v = nn.Linear(embed_dim, embed_dim, bias=False)
            o = nn.Linear(embed_dim, embed_dim, bias=False)
            if moe_experts:
                # the MoE variant (oracle/moe.py): router + experts replace the dense FFN
                from .moe import OracleMoE
                mlp = OracleMoE(embed_dim, d_ff, moe_experts, moe_capacity)
            else:
                gate = nn.Linear(embed_dim, d_ff, bias=False)
                down = nn.Linear(d_ff, embed_dim, bias=False)
                up = nn.Linear(embed_dim, d_ff, bias=False)
                mlp = FeedForward(gate, down, up)
            self.layers.append(Layer(Attention(q, k, v, o, num_heads, head_dim), mlp, RMSNorm(embed_dim),
                                     RMSNorm(embed_dim)))
        self.norm = RMSNorm(embed_dim)
        self.board_head = nn.Linear(embed_dim, BOARD_VOCAB_SIZE)
        self.policy_head = nn.Linear(embed_dim, MOVE_VOCAB_SIZE)
        self.thinking_policy_head = nn.Linear(embed_dim, MOVE_VOCAB_SIZE)
        self.wl_head = ValueHead(embed_dim, n_buckets, value_hidden_size)
        self.d_head = ValueHead(embed_dim, n_buckets, value_hidden_size)
        self.fourier_encoder = FourierEncoder(embed_dim, num_fourier_freq)
        self.register_buffer("wl_bucket_centers", make_wl_buckets(n_buckets, wl_sigma))
        self.register_buffer("d_bucket_centers", make_d_buckets(n_buckets))

    def _layer(self, layer, x, mask, input_pos):
        B, S, E = x.shape
        h = layer.sa_norm(x)
        a = layer.attn
        q = a.q_proj(h).view(B, S, a.num_heads, a.head_dim)
        k = a.k_proj(h).view(B, S, a.num_heads, a.head_dim)
        v = a.v_proj(h).view(B, S, a.num_heads, a.head_dim)
        q = apply_rope(q, self.rope, input_pos).transpose(1, 2)
        k = apply_rope(k, self.rope, input_pos).transpose(1, 2)
        v = v.transpose(1, 2)
        if mask is None:
            o = F.scaled_dot_product_attention(q, k, v, is_causal=True)
        else:
            o = F.scaled_dot_product_attention(q, k, v, attn_mask=mask[:, None])
        x = x + a.output_proj(o.transpose(1, 2).reshape(B, S, E))
        return x + layer.mlp(layer.mlp_norm(x))

    def forward(self, x, input_pos=None, mask_type="causal", block_id=None, wl_values=None, d_values=None,
                wl_positions=None, d_positions=None):
        B, S = x.shape
        if input_pos is None:
            input_pos = torch.arange(S, device=x.device).unsqueeze(0)
        if mask_type == "causal":
            mask = None
        else:
            if block_id is None:
                raise ValueError("block_id is required for prefix mask mode")
            causal = torch.tril(torch.ones(S, S, device=x.device, dtype=torch.bool))
            mask = causal.unsqueeze(0) | (block_id.unsqueeze(-1) == block_id.unsqueeze(-2))
        h = self.tok_embedding(x)
        if wl_positions is not None and wl_positions.any():
            h[wl_positions] = self.fourier_encoder(wl_values[wl_positions]).to(h.dtype)
        if d_positions is not None and d_positions.any():
            h[d_positions] = self.fourier_encoder(d_values[d_positions]).to(h.dtype)
        for layer in self.layers:
            h = self._layer(layer, h, mask, input_pos)
        return self.norm(h)

    def discretize_to_bucket(self, values, bucket_centers):
        """model.py:189-194."""
        idx = (values.unsqueeze(-1) - bucket_centers.unsqueeze(0)).abs().argmin(dim=-1)
        return bucket_centers[idx]
