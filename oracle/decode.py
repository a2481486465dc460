"""CPU oracle for the KV-cache inference backbone (test infrastructure only:
imported by tests/, never by the product path).

Restates, in numpy fp32:

* ``forward``: chessdecoder/export/backbone_causal.py:77-150
  (``BackboneCausal.forward``): token embedding with the Fourier override
  blended in (lines 99-103, encoder at 55-59), per layer RMSNorm (61-64),
  q / k / v projections with RoPE at explicit positions (66-75), attention over
  past + new keys with the additive mask (121-134), output projection +
  residual, SwiGLU MLP + residual (139-143), final RMSNorm (145);
* ``Batched``: the cache and mask bookkeeping of
  chessdecoder/cpp/decoder/batched_backbone.cpp (causalForward 117-158,
  causalIncremental 160-177, prefixForward 192-205, prefixIncremental 207-225,
  prefixBlockForward 227-258, probes 264-305, mark helpers 74-104);
* ``chess_decoder_to_module``: the weight mapping of backbone_causal.py:153-188
  (``from_chess_decoder``), in reverse.

Pinned by tests/golden/decode_reference.pt, produced by the reference's own
``BackboneCausal`` module (tests/golden/make_decode_golden.py).
"""
from __future__ import annotations

import numpy as np

NEG = -1e9


def module_to_chess_decoder(w: dict, num_layers: int) -> dict:
    """BackboneCausal parameter names -> ChessDecoder ``state_dict`` names
    (backbone_causal.py:171-186 read the other way)."""
    out = {"tok_embedding.weight": w["tok_embedding.weight"],
           "fourier_encoder.frequencies": w["fourier_frequencies"],
           "fourier_encoder.proj.weight": w["fourier_proj.weight"],
           "fourier_encoder.proj.bias": w["fourier_proj.bias"],
           "norm.scale": w["final_norm_weight"]}
    for i in range(num_layers):
        p = f"layers.{i}."
        out[p + "attn.q_proj.weight"] = w[f"q_projs.{i}.weight"]
        out[p + "attn.k_proj.weight"] = w[f"k_projs.{i}.weight"]
        out[p + "attn.v_proj.weight"] = w[f"v_projs.{i}.weight"]
        out[p + "attn.output_proj.weight"] = w[f"o_projs.{i}.weight"]
        out[p + "sa_norm.scale"] = w[f"sa_norm_weights.{i}"]
        out[p + "mlp_norm.scale"] = w[f"mlp_norm_weights.{i}"]
        out[p + "mlp.w1.weight"] = w[f"gate_projs.{i}.weight"]
        out[p + "mlp.w3.weight"] = w[f"up_projs.{i}.weight"]
        out[p + "mlp.w2.weight"] = w[f"down_projs.{i}.weight"]
    return out


def rope_table(max_seq_len: int, head_dim: int, base: float = 10000.0) -> np.ndarray:
    """[max_seq_len, head_dim / 2, 2] = (cos, sin) of p * base^(-2i / head_dim)."""
    theta = 1.0 / (base ** (np.arange(0, head_dim, 2, dtype=np.float32)[: head_dim // 2] / head_dim))
    ang = np.outer(np.arange(max_seq_len, dtype=np.float32), theta.astype(np.float32))
    return np.stack([np.cos(ang), np.sin(ang)], axis=-1).astype(np.float32)


def _rms(x, w):
    return x / np.sqrt((x * x).mean(-1, keepdims=True) + 1e-6) * w


def _rope(x, pos, table):
    """x [B, S, H, D], pos [B, S]: interleaved pairs rotated by table[pos]."""
    cs = table[pos][:, :, None]  # [B, S, 1, D/2, 2]
    xr = x.reshape(*x.shape[:-1], -1, 2)
    a, b = xr[..., 0], xr[..., 1]
    c, s = cs[..., 0], cs[..., 1]
    return np.stack([a * c - b * s, b * c + a * s], axis=-1).reshape(x.shape)


def forward(w: dict, cfg: dict, ids, pos, mask, past_k, past_v, ov, om, rope):
    """BackboneCausal.forward on numpy arrays (ChessDecoder weight names).
    ids / pos [B, S] int, mask [B, 1, S, P + S] additive, past_k / past_v
    [L, B, H, P, D], ov [B, S] float, om [B, S] bool.  Returns (hidden [B, S, E],
    present_k, present_v)."""
    L, H, E = cfg["num_layers"], cfg["num_heads"], cfg["embed_dim"]
    D = E // H
    B, S = ids.shape
    h = w["tok_embedding.weight"][ids].astype(np.float32)
    f = 2 * np.pi * ov.reshape(-1, 1).astype(np.float32) * w["fourier_encoder.frequencies"]
    feat = np.concatenate([np.cos(f), np.sin(f)], axis=-1)
    four = (feat @ w["fourier_encoder.proj.weight"].T + w["fourier_encoder.proj.bias"]).reshape(B, S, E)
    h = np.where(om[..., None], four, h).astype(np.float32)
    pk, pv = [], []
    for i in range(L):
        p = f"layers.{i}."
        n = _rms(h, w[p + "sa_norm.scale"])
        q = (n @ w[p + "attn.q_proj.weight"].T).reshape(B, S, H, D)
        k = (n @ w[p + "attn.k_proj.weight"].T).reshape(B, S, H, D)
        v = (n @ w[p + "attn.v_proj.weight"].T).reshape(B, S, H, D)
        q, k = _rope(q, pos, rope), _rope(k, pos, rope)
        q, k, v = q.transpose(0, 2, 1, 3), k.transpose(0, 2, 1, 3), v.transpose(0, 2, 1, 3)
        k = np.concatenate([past_k[i], k], axis=2)
        v = np.concatenate([past_v[i], v], axis=2)
        pk.append(k)
        pv.append(v)
        s = q @ k.transpose(0, 1, 3, 2) / np.sqrt(D) + mask
        s = s - s.max(-1, keepdims=True)
        pr = np.exp(s)
        pr /= pr.sum(-1, keepdims=True)
        a = (pr @ v).transpose(0, 2, 1, 3).reshape(B, S, E)
        h = a @ w[p + "attn.output_proj.weight"].T + h
        n = _rms(h, w[p + "mlp_norm.scale"])
        g = n @ w[p + "mlp.w1.weight"].T
        u = n @ w[p + "mlp.w3.weight"].T
        h = (g / (1 + np.exp(-g)) * u) @ w[p + "mlp.w2.weight"].T + h
    return _rms(h, w["norm.scale"]).astype(np.float32), np.stack(pk), np.stack(pv)


class Batched:
    """BatchedBackbone's caches (growing K / V, one additive mask buffer per
    cache) around ``forward``.  Tensors in and out are numpy arrays."""

    def __init__(self, w: dict, cfg: dict, B: int, max_len: int):
        self.w, self.cfg, self.B, self.max_len = w, cfg, B, max_len
        L, H = cfg["num_layers"], cfg["num_heads"]
        D = cfg["embed_dim"] // H
        self.rope = rope_table(max(max_len, cfg.get("max_seq_len", max_len)), D)
        self.empty = np.zeros((L, B, H, 0, D), np.float32)
        self.ck = self.cv = self.pk = self.pv = self.empty
        self.cbuf = np.full((B, max_len), NEG, np.float32)
        self.pbuf = np.full((B, max_len), NEG, np.float32)

    @property
    def causal_len(self):
        return self.ck.shape[3]

    @property
    def prefix_len(self):
        return self.pk.shape[3]

    def _run(self, ids, pos, mask, k, v, ov, om):
        return forward(self.w, self.cfg, np.asarray(ids), np.asarray(pos), mask, k, v, np.asarray(ov, np.float32),
                       np.asarray(om, bool), self.rope)

    def _cached_mask(self, buf, old, S):
        B = self.B
        m = np.full((B, 1, S, old + S), NEG, np.float32)
        m[..., :old] = buf[:, None, None, :old]
        return m

    def causal_forward(self, ids, pos, ov, om, active, num_real):
        S = np.asarray(ids).shape[1]
        old = self.causal_len
        m = self._cached_mask(self.cbuf, old, S)
        j = np.arange(S)
        new_valid = j[None, :] < np.asarray(num_real)[:, None]
        att = new_valid[:, None, :] & (j[None, :] <= j[:, None])[None]
        m[..., old:] = np.where(att, 0.0, NEG)[:, None]
        h, self.ck, self.cv = self._run(ids, pos, m, self.ck, self.cv, ov, om)
        self.cbuf[:, old:old + S][new_valid] = 0.0
        return h

    def _incremental(self, buf, k, v, ids, pos, ov, om, active):
        new = k.shape[3]
        buf[np.asarray(active, bool), new] = 0.0
        m = buf[:, None, None, :new + 1].copy()
        return self._run(ids, pos, m, k, v, ov, om)

    def causal_incremental(self, ids, pos, ov, om, active):
        h, self.ck, self.cv = self._incremental(self.cbuf, self.ck, self.cv, ids, pos, ov, om, active)
        return h

    def prefix_forward(self, ids, pos, mask, ov, om, active):
        S = np.asarray(ids).shape[1]
        h, self.pk, self.pv = self._run(ids, pos, np.asarray(mask, np.float32), self.pk, self.pv, ov, om)
        self.pbuf[np.asarray(active, bool), :S] = 0.0
        return h

    def prefix_incremental(self, ids, pos, ov, om, active):
        h, self.pk, self.pv = self._incremental(self.pbuf, self.pk, self.pv, ids, pos, ov, om, active)
        return h

    def prefix_block_forward(self, ids, pos, ov, om, active):
        S = np.asarray(ids).shape[1]
        old = self.prefix_len
        act = np.asarray(active, bool)
        m = self._cached_mask(self.pbuf, old, S)
        m[..., old:] = np.where(act, 0.0, NEG)[:, None, None, None]
        h, self.pk, self.pv = self._run(ids, pos, m, self.pk, self.pv, ov, om)
        self.pbuf[act, old:old + S] = 0.0
        return h

    def _probe(self, buf, k, v, ids, pos, ov, om):
        S = np.asarray(ids).shape[1]
        old = k.shape[3]
        m = self._cached_mask(buf, old, S)
        m[..., old:] = 0.0
        return self._run(ids, pos, m, k, v, ov, om)[0]

    def causal_probe(self, ids, pos, ov, om):
        return self._probe(self.cbuf, self.ck, self.cv, ids, pos, ov, om)

    def prefix_probe(self, ids, pos, ov, om):
        return self._probe(self.pbuf, self.pk, self.pv, ids, pos, ov, om)
