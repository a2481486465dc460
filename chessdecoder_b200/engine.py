"""The B200 training step for ChessDecoder: parameter store, fused two-pass
forward, fused heads and losses, explicit backward and the optimizer step.

This replaces the body of the reference loop, chessdecoder/train/train.py:157-253:

* both passes run as ONE batch of 2B sequences (rows [0, B*S) causal = pass 1,
  rows [B*S, 2B*S) prefix = pass 2).  They share weights and inputs, so every
  GEMM is twice as tall and every weight is read once per step instead of
  twice; the attention kernel applies the causal or the block-prefix mask per
  sequence;
* heads run only where the loss looks: the board head on pass-1 rows, the
  policy head on the gathered move rows, the value heads on gathered WL / D
  rows (the reference computes policy logits at every position);
* the backward is written out by hand (no autograd): weight gradients land in
  one flat fp32 buffer laid out in the order the backward finishes them, so a
  data-parallel all-reduce can start on a finished layer while the next one is
  still being differentiated;
* AdamW, the global-norm clip and the bf16 shadow weights are one kernel over
  the flat buffers.

Tensors named *_16 are bf16, everything else fp32 unless stated.
"""
from __future__ import annotations

import dataclasses
import math
from typing import Callable, Optional

import numpy as np
import torch

from . import kernels as K
from . import vocab as V

IGNORE_INDEX = -100


@dataclasses.dataclass
class ModelConfig:
    """The ``model:`` section of chessdecoder/train/config.yaml (plus vocab size)."""
    vocab_size: int = V.vocab_size
    embed_dim: int = 1024
    num_heads: int = 16
    num_layers: int = 12
    max_seq_len: int = 256
    d_ff: Optional[int] = 1536
    n_buckets: int = 100
    value_hidden_size: int = 256
    num_fourier_freq: int = 128
    wl_sigma: float = 0.4
    moe_experts: int = 0        # MoE variant: experts per layer (0 = the dense SwiGLU MLP)
    moe_capacity: float = 1.25  # capacity factor (slots per expert = ceil(cf * 2 * tokens / experts))
    finetune: bool = False      # finetune step: the thinking head is trained (chessdecoder/finetune/train.py)

    @property
    def head_dim(self):
        return self.embed_dim // self.num_heads

    @property
    def ff(self):
        return self.d_ff if self.d_ff is not None else 4 * self.embed_dim


def make_wl_buckets(n_buckets=100, sigma=0.4):
    """chessdecoder/models/model.py:12-16."""
    t = torch.linspace(0.5 / n_buckets, 1 - 0.5 / n_buckets, n_buckets)
    return (sigma * math.sqrt(2) * torch.erfinv(2 * t - 1)).clamp(-1.0, 1.0)


def make_d_buckets(n_buckets=100):
    """chessdecoder/models/model.py:19-21."""
    return torch.linspace(0.5 / n_buckets, 1 - 0.5 / n_buckets, n_buckets)


def rope_table(max_seq_len: int, dim: int, base: float = 10000.0) -> torch.Tensor:
    """RoPE cache [max_seq_len, dim/2, 2] = (cos, sin) of p * base^(-2i/dim)
    (torchtune RotaryPositionalEmbeddings, used at chessdecoder/models/model.py:87)."""
    theta = 1.0 / (base ** (torch.arange(0, dim, 2)[: dim // 2].float() / dim))
    ang = torch.einsum("i,j->ij", torch.arange(max_seq_len, dtype=theta.dtype), theta).float()
    return torch.stack([torch.cos(ang), torch.sin(ang)], dim=-1).contiguous()


# ---------------------------------------------------------------------------
# Parameter store
# ---------------------------------------------------------------------------
def param_specs(cfg: ModelConfig):
    """(name, shape) of every trainable parameter, in flat-buffer order: the
    order in which the backward produces final gradients (heads, final norm,
    layers last to first, Fourier encoder, embedding)."""
    E, F, L = cfg.embed_dim, cfg.ff, cfg.num_layers
    hv, nb, nf = cfg.value_hidden_size, cfg.n_buckets, cfg.num_fourier_freq
    specs = [("board_head.weight", (V.board_vocab_size, E)), ("board_head.bias", (V.board_vocab_size,)),
             ("policy_head.weight", (V.move_vocab_size, E)), ("policy_head.bias", (V.move_vocab_size,))]
    if cfg.finetune:  # trained only by the finetune step; pretraining leaves it out of AdamW
        specs += [("thinking_policy_head.weight", (V.move_vocab_size, E)),
                  ("thinking_policy_head.bias", (V.move_vocab_size,))]
    for h in ("wl_head", "d_head"):
        specs += [(f"{h}.mlp.0.weight", (hv, E)), (f"{h}.mlp.0.bias", (hv,)), (f"{h}.mlp.2.weight", (nb, hv)),
                  (f"{h}.mlp.2.bias", (nb,))]
    specs.append(("norm.scale", (E,)))
    X = cfg.moe_experts
    for i in reversed(range(L)):
        # per layer the MLP block (its gradients are final first) then the attention block
        p = f"layers.{i}."
        if X:
            specs += [(p + "mlp.router.weight", (X, E)), (p + "mlp.experts.w13", (X, 2 * F, E)),
                      (p + "mlp.experts.w2", (X, E, F))]
        else:
            specs += [(p + "mlp.w1.weight", (F, E)), (p + "mlp.w3.weight", (F, E)), (p + "mlp.w2.weight", (E, F))]
        specs += [(p + "mlp_norm.scale", (E,))]
        specs += [(p + "attn.q_proj.weight", (E, E)), (p + "attn.k_proj.weight", (E, E)),
                  (p + "attn.v_proj.weight", (E, E)), (p + "attn.output_proj.weight", (E, E))]
        specs += [(p + "sa_norm.scale", (E,))]
    specs += [("fourier_encoder.frequencies", (1, nf)), ("fourier_encoder.proj.weight", (E, 2 * nf)),
              ("fourier_encoder.proj.bias", (E,)), ("tok_embedding.weight", (cfg.vocab_size, E))]
    return specs


def reference_param_names(cfg: ModelConfig):
    """Parameter names in the order of the reference model's ``parameters()``
    (its construction order, chessdecoder/models/model.py:84-132: embedding;
    per layer q, k, v, output projections, w1, w2, w3 (or the MoE variant's
    router and experts), sa_norm, mlp_norm; final norm; board, policy and
    thinking heads; WL / D value heads; Fourier encoder) -- the indices of a
    ``torch.optim`` optimizer's ``state_dict`` built on those parameters."""
    names = ["tok_embedding.weight"]
    for i in range(cfg.num_layers):
        p = f"layers.{i}."
        names += [p + f"attn.{n}.weight" for n in ("q_proj", "k_proj", "v_proj", "output_proj")]
        if cfg.moe_experts:
            names += [p + "mlp.router.weight", p + "mlp.experts.w13", p + "mlp.experts.w2"]
        else:
            names += [p + "mlp.w1.weight", p + "mlp.w2.weight", p + "mlp.w3.weight"]
        names += [p + "sa_norm.scale", p + "mlp_norm.scale"]
    names.append("norm.scale")
    for h in ("board_head", "policy_head", "thinking_policy_head"):
        names += [h + ".weight", h + ".bias"]
    for h in ("wl_head", "d_head"):
        names += [f"{h}.mlp.0.weight", f"{h}.mlp.0.bias", f"{h}.mlp.2.weight", f"{h}.mlp.2.bias"]
    names += ["fourier_encoder.frequencies", "fourier_encoder.proj.weight", "fourier_encoder.proj.bias"]
    return names


# Tensors that must stay adjacent (fused GEMM operands): q|k|v and w1|w3.
_ALIGN = 64  # elements: every parameter starts on a 256-byte boundary


def flat_layout(cfg: ModelConfig):
    """({name: (offset, shape, numel)}, total elements) of the flat parameter
    buffers: param_specs order, every tensor 256-byte aligned except that
    q|k|v and w1|w3 are packed back to back so the fused projections read one
    [3E, E] / [2F, E] matrix."""
    offsets = {}
    off = 0
    for name, shape in param_specs(cfg):
        n = int(np.prod(shape))
        offsets[name] = (off, shape, n)
        pad = 0 if name.endswith(("q_proj.weight", "k_proj.weight", "mlp.w1.weight")) else _ALIGN
        off += n if pad == 0 else (n + _ALIGN - 1) // _ALIGN * _ALIGN
    return offsets, off


class ParamStore:
    """All trainable parameters in one flat fp32 buffer, with matching flat
    gradient, AdamW moment and bf16 shadow buffers.  ``param(name)`` returns a
    view shaped like the reference parameter."""

    def __init__(self, cfg: ModelConfig, device, optimizer_state: bool = True):
        self.cfg = cfg
        self.device = torch.device(device)
        self.offsets, off = flat_layout(cfg)
        self.numel = off
        self.flat = torch.zeros(off, dtype=torch.float32, device=self.device)
        self.flat16 = torch.zeros(off, dtype=torch.bfloat16, device=self.device)
        if optimizer_state:
            self.grad = torch.zeros(off, dtype=torch.float32, device=self.device)
            self.exp_avg = torch.zeros(off, dtype=torch.float32, device=self.device)
            self.exp_avg_sq = torch.zeros(off, dtype=torch.float32, device=self.device)
        else:  # the nn.Module front end: gradients are allocated per backward, moments by the optimizer
            self.grad = self.exp_avg = self.exp_avg_sq = None
        self.step = 0
        # the thinking head gets no gradient in pretraining (train.py never calls
        # it): kept outside the flat buffers unless the finetune step trains it
        E = cfg.embed_dim
        self.thinking_weight = torch.zeros(V.move_vocab_size, E, device=self.device)
        self.thinking_bias = torch.zeros(V.move_vocab_size, device=self.device)

    def names(self):
        return list(self.offsets)

    def _view(self, buf, name):
        off, shape, n = self.offsets[name]
        return buf[off:off + n].view(shape)

    def param(self, name):
        return self._view(self.flat, name)

    def grad_of(self, name):
        return self._view(self.grad, name)

    def bf16(self, name):
        return self._view(self.flat16, name)

    def span(self, first: str, last: str, buf=None):
        """Contiguous view from the start of `first` through the end of `last`."""
        buf = self.flat16 if buf is None else buf
        o0 = self.offsets[first][0]
        o1, _, n1 = self.offsets[last]
        return buf[o0:o1 + n1]

    def refresh_bf16(self):
        K.cast_bf16(self.flat, self.flat16)

    # -- state dict in the reference layout ---------------------------------
    def load_state_dict(self, sd: dict):
        with torch.no_grad():
            for name in self.offsets:
                self.param(name).copy_(sd[name].reshape(self.offsets[name][1]))
            if "thinking_policy_head.weight" in sd and "thinking_policy_head.weight" not in self.offsets:
                self.thinking_weight.copy_(sd["thinking_policy_head.weight"])
                self.thinking_bias.copy_(sd["thinking_policy_head.bias"])
        self.refresh_bf16()

    def state_dict(self) -> dict:
        sd = {name: self.param(name).detach().clone() for name in self.offsets}
        if "thinking_policy_head.weight" not in self.offsets:
            sd["thinking_policy_head.weight"] = self.thinking_weight.clone()
            sd["thinking_policy_head.bias"] = self.thinking_bias.clone()
        return sd

    # -- AdamW state in torch.optim.AdamW's state_dict layout ------------------
    def optimizer_state_dict(self, lr, betas, eps, weight_decay) -> dict:
        """The moments and step count as ``torch.optim.AdamW(model.parameters())
        .state_dict()`` holds them (per-parameter index in the reference model's
        parameter order; parameters that never had a step -- the thinking head
        in pretraining -- have no entry), so a reference checkpoint's optimizer
        can resume from it and the other way round."""
        names = reference_param_names(self.cfg)
        state = {}
        if self.step > 0:
            for i, n in enumerate(names):
                if n in self.offsets:
                    state[i] = {"step": torch.tensor(float(self.step)),
                                "exp_avg": self._view(self.exp_avg, n).detach().clone(),
                                "exp_avg_sq": self._view(self.exp_avg_sq, n).detach().clone()}
        group = {"lr": lr, "betas": tuple(betas), "eps": eps, "weight_decay": weight_decay, "amsgrad": False,
                 "maximize": False, "foreach": None, "capturable": False, "differentiable": False, "fused": None,
                 "decoupled_weight_decay": True, "params": list(range(len(names)))}
        return {"state": state, "param_groups": [group]}

    def load_optimizer_state_dict(self, sd: dict):
        """Moments and step count from an AdamW state_dict in the reference
        parameter order (see ``optimizer_state_dict``).  Returns the param
        group (its lr, betas, eps, weight_decay)."""
        names = reference_param_names(self.cfg)
        if len(sd["param_groups"]) != 1 or len(sd["param_groups"][0]["params"]) != len(names):
            raise ValueError("optimizer state_dict does not match this model's parameters")
        steps = set()
        with torch.no_grad():
            self.exp_avg.zero_()
            self.exp_avg_sq.zero_()
            for i, st in sd["state"].items():
                n = names[int(i)]
                if n not in self.offsets:
                    continue  # e.g. a trained thinking head: pretraining leaves it out of AdamW
                self._view(self.exp_avg, n).copy_(st["exp_avg"].reshape(self.offsets[n][1]))
                self._view(self.exp_avg_sq, n).copy_(st["exp_avg_sq"].reshape(self.offsets[n][1]))
                steps.add(int(float(st["step"])))
        if len(steps) > 1:
            raise ValueError(f"parameters at different AdamW steps {sorted(steps)}: one shared step count expected")
        self.step = steps.pop() if steps else 0
        return sd["param_groups"][0]

    def layer_grad_span(self, i: int, part: Optional[str] = None):
        """[start, end) of layer i's gradients in the flat buffer; part "mlp"
        (the MLP block and its norm, final first in the backward) or "attn"
        (the attention block and its norm)."""
        p = f"layers.{i}."
        first_mlp = p + ("mlp.router.weight" if self.cfg.moe_experts else "mlp.w1.weight")
        s = self.offsets[first_mlp][0]
        m = self.offsets[p + "attn.q_proj.weight"][0]
        o, _, n = self.offsets[p + "sa_norm.scale"]
        e = (o + n + _ALIGN - 1) // _ALIGN * _ALIGN
        if part == "mlp":
            return s, m
        if part == "attn":
            return m, e
        return s, e


def init_reference_weights(cfg: ModelConfig, seed: int = 0) -> dict:
    """Initial weights exactly as ``torch.manual_seed(seed); ChessDecoder(...)``
    draws them (construction order of chessdecoder/models/model.py:84-132:
    embedding N(0,1); per layer q,k,v,o then gate,down,up with nn.Linear's
    kaiming-uniform init; norms = 1; board, policy, thinking heads; WL / D value
    heads; Fourier frequencies N(0,1) then projection)."""
    import torch.nn as nn
    g = torch.random.fork_rng(devices=[])  # weights are drawn on the CPU generator only
    with g:
        torch.manual_seed(seed)
        E, F, L = cfg.embed_dim, cfg.ff, cfg.num_layers
        sd = {}
        sd["tok_embedding.weight"] = nn.Embedding(cfg.vocab_size, E).weight.data
        for i in range(L):
            p = f"layers.{i}."
            for n in ("q_proj", "k_proj", "v_proj", "output_proj"):
                sd[p + f"attn.{n}.weight"] = nn.Linear(E, E, bias=False).weight.data
            if cfg.moe_experts:
                # router, then per expert gate / down / up (oracle/moe.py construction order)
                sd[p + "mlp.router.weight"] = nn.Linear(E, cfg.moe_experts, bias=False).weight.data
                w13, w2 = [], []
                for _ in range(cfg.moe_experts):
                    gate = nn.Linear(E, F, bias=False).weight.data
                    down = nn.Linear(F, E, bias=False).weight.data
                    up = nn.Linear(E, F, bias=False).weight.data
                    w13.append(torch.cat([gate, up], 0))
                    w2.append(down)
                sd[p + "mlp.experts.w13"] = torch.stack(w13)
                sd[p + "mlp.experts.w2"] = torch.stack(w2)
            else:
                sd[p + "mlp.w1.weight"] = nn.Linear(E, F, bias=False).weight.data
                sd[p + "mlp.w2.weight"] = nn.Linear(F, E, bias=False).weight.data
                sd[p + "mlp.w3.weight"] = nn.Linear(E, F, bias=False).weight.data
            sd[p + "sa_norm.scale"] = torch.ones(E)
            sd[p + "mlp_norm.scale"] = torch.ones(E)
        sd["norm.scale"] = torch.ones(E)
        for name, n in (("board_head", V.board_vocab_size), ("policy_head", V.move_vocab_size),
                        ("thinking_policy_head", V.move_vocab_size)):
            lin = nn.Linear(E, n)
            sd[name + ".weight"], sd[name + ".bias"] = lin.weight.data, lin.bias.data
        for h in ("wl_head", "d_head"):
            l0 = nn.Linear(E, cfg.value_hidden_size)
            l2 = nn.Linear(cfg.value_hidden_size, cfg.n_buckets)
            sd[h + ".mlp.0.weight"], sd[h + ".mlp.0.bias"] = l0.weight.data, l0.bias.data
            sd[h + ".mlp.2.weight"], sd[h + ".mlp.2.bias"] = l2.weight.data, l2.bias.data
        sd["fourier_encoder.frequencies"] = torch.randn(1, cfg.num_fourier_freq)
        lp = nn.Linear(2 * cfg.num_fourier_freq, E)
        sd["fourier_encoder.proj.weight"], sd["fourier_encoder.proj.bias"] = lp.weight.data, lp.bias.data
    return sd


# ---------------------------------------------------------------------------
# Batch preparation (host side: index lists, loss normalisers)
# ---------------------------------------------------------------------------
@dataclasses.dataclass
class DeviceBatch:
    B: int
    S: int
    ids: torch.Tensor            # int64 [B*S]
    wl_t: torch.Tensor           # f32 [B*S]
    d_t: torch.Tensor            # f32 [B*S]
    wl_pos: torch.Tensor         # u8 [B*S]
    d_pos: torch.Tensor          # u8 [B*S]
    slot: torch.Tensor           # i32 [B*S]   Fourier slot or -1
    frows: torch.Tensor          # i32 [Nf]    token rows of the Fourier slots
    bid: torch.Tensor            # i32 [B, S]
    board_t: torch.Tensor        # i32 [B*S]
    board_w: torch.Tensor        # f32 [B*S]
    prow: torch.Tensor           # i32 [Nm]    merged-batch rows of the policy head (pass 2)
    pt: torch.Tensor             # i32 [Nm]
    wrow: torch.Tensor           # i32 [Nw]
    wtgt: torch.Tensor           # f32 [Nw]
    wvalid: torch.Tensor         # f32 [Nw]
    drow: torch.Tensor           # i32 [Nd]
    dtgt: torch.Tensor           # f32 [Nd]
    dvalid: torch.Tensor         # f32 [Nd]
    norms: torch.Tensor          # f32 [5] = 1/(count+1e-8) for move, board, wl, d, thinking move (0 when the loss is 0)
    trow: Optional[torch.Tensor] = None  # i32 [Nt]  merged-batch rows of the thinking head (finetune)
    tt: Optional[torch.Tensor] = None    # i32 [Nt]
    h2d_bytes: int = 0


def _host_index_lists(b: dict, require_pairing: bool = True):
    """Numpy restatement of the index bookkeeping of train.py:180-233.

    The D head reads rows at wl_positions with targets at d_positions, zipped
    in order (train.py:225-230); unequal counts are an error there, and here
    unless ``require_pairing`` is False (forward-only use), in which case the
    D rows are cut to the shorter list.

    A batch with ``thinking_move_mask`` is a finetune batch
    (chessdecoder/finetune/train.py:287-346): the board mask starts at the
    first move of either kind, the thinking head reads the thinking rows, and
    the WL head reads stm+1 of every move row of either kind."""
    ids = b["input_ids"].numpy()
    Bn, S = ids.shape
    move_mask = b["move_mask"].numpy()
    wl_pos = b["wl_positions"].numpy()
    d_pos = b["d_positions"].numpy()
    board_t = b["board_target_ids"].numpy()
    move_t = b["move_target_ids"].numpy()
    wl_t = b["wl_targets"].numpy().astype(np.float32)
    d_t = b["d_targets"].numpy().astype(np.float32)
    valid = b["wdl_valid"].numpy()
    BS = Bn * S
    # board mask: target != -100 and position >= first move (train.py:183-191)
    think = b["thinking_move_mask"].numpy() if "thinking_move_mask" in b else np.zeros_like(move_mask)
    any_move = move_mask | think
    has = any_move.any(1)
    first = np.where(has, any_move.argmax(1), S)
    board_mask = (board_t != IGNORE_INDEX) & (np.arange(S)[None, :] >= first[:, None])
    # Fourier slots: every WL or D placeholder
    fmask = (wl_pos | d_pos).reshape(-1)
    frows = np.nonzero(fmask)[0].astype(np.int32)
    slot = np.full(BS, -1, dtype=np.int32)
    slot[frows] = np.arange(frows.size, dtype=np.int32)
    # policy rows (pass 2 = second half of the merged batch)
    mflat = np.nonzero(move_mask.reshape(-1))[0]
    prow = (BS + mflat).astype(np.int32)
    pt = move_t.reshape(-1)[mflat].astype(np.int32)
    # thinking-head rows (finetune) in the same merged-batch layout
    tflat = np.nonzero(think.reshape(-1))[0]
    trow = (BS + tflat).astype(np.int32)
    tt = move_t.reshape(-1)[tflat].astype(np.int32)
    # WL rows at stm + 1 (clamped), targets copied to stm by the loader
    bb, ss = np.nonzero(any_move)
    wrow = (BS + bb * S + np.minimum(ss + 1, S - 1)).astype(np.int32)
    wtgt = wl_t[bb, ss]
    wvalid = valid[bb, ss].astype(np.float32)
    # D rows at WL positions, targets at D positions (zipped in row-major order)
    wpf = np.nonzero(wl_pos.reshape(-1))[0]
    dpf = np.nonzero(d_pos.reshape(-1))[0]
    if wpf.size != dpf.size:
        if require_pairing:
            raise ValueError("wl_positions and d_positions must pair up one to one (train.py:225-230)")
        k = min(wpf.size, dpf.size)
        wpf, dpf = wpf[:k], dpf[:k]
    drow = (BS + wpf).astype(np.int32)
    dtgt = d_t.reshape(-1)[dpf]
    dvalid = valid.reshape(-1)[dpf].astype(np.float32)
    nb = board_mask.sum()
    norms = np.array([
        1.0 / (mflat.size + 1e-8),
        1.0 / (nb + 1e-8),
        (1.0 / (wvalid.sum() + 1e-8)) if (wvalid.size and wvalid.sum() > 0) else 0.0,
        (1.0 / (dvalid.sum() + 1e-8)) if (dvalid.size and dvalid.sum() > 0) else 0.0,
        1.0 / (tflat.size + 1e-8),
    ], dtype=np.float32)
    board_t32 = np.where(board_mask, board_t, IGNORE_INDEX).reshape(-1).astype(np.int32)
    return dict(ids=ids.reshape(-1).astype(np.int64), wl_t=wl_t.reshape(-1), d_t=d_t.reshape(-1),
                wl_pos=wl_pos.reshape(-1).astype(np.uint8), d_pos=d_pos.reshape(-1).astype(np.uint8), slot=slot,
                frows=frows, bid=b["block_id"].numpy().astype(np.int32), board_t=board_t32,
                board_w=board_mask.reshape(-1).astype(np.float32), prow=prow, pt=pt, trow=trow, tt=tt, wrow=wrow,
                wtgt=wtgt.astype(np.float32), wvalid=wvalid, drow=drow, dtgt=dtgt.astype(np.float32), dvalid=dvalid,
                norms=norms), Bn, S


def prepare_batch(batch: dict, device, require_pairing: bool = True) -> DeviceBatch:
    """Builds the device batch: index lists on the host (numpy), then one
    pinned host buffer per dtype and one host-to-device copy each."""
    host = {k: (v.cpu() if torch.is_tensor(v) else torch.as_tensor(v)) for k, v in batch.items()}
    lists, Bn, S = _host_index_lists(host, require_pairing)
    groups = {"i64": ["ids"], "f32": ["wl_t", "d_t", "board_w", "wtgt", "wvalid", "dtgt", "dvalid", "norms"],
              "i32": ["slot", "frows", "bid", "board_t", "prow", "pt", "trow", "tt", "wrow", "drow"],
              "u8": ["wl_pos", "d_pos"]}
    dt = {"i64": torch.int64, "f32": torch.float32, "i32": torch.int32, "u8": torch.uint8}
    out = {}
    total = 0
    for g, names in groups.items():
        sizes = [lists[n].size for n in names]
        # 16-byte aligned segments
        align = 16 // torch.empty(0, dtype=dt[g]).element_size()
        offs, o = [], 0
        for s in sizes:
            offs.append(o)
            o += (s + align - 1) // align * align
        hbuf = torch.empty(max(o, 1), dtype=dt[g], pin_memory=torch.cuda.is_available())
        hv = hbuf.numpy()
        for n, off, s in zip(names, offs, sizes):
            hv[off:off + s] = lists[n].reshape(-1)
        dbuf = hbuf.to(device, non_blocking=True)
        total += hbuf.numel() * hbuf.element_size()
        for n, off, s in zip(names, offs, sizes):
            out[n] = dbuf[off:off + s]
    out["bid"] = out["bid"].view(Bn, S)
    return DeviceBatch(B=Bn, S=S, h2d_bytes=total, **out)


# ---------------------------------------------------------------------------
# Backbone (embedding output -> final RMSNorm), forward and backward
# ---------------------------------------------------------------------------
class LayerSaved:
    __slots__ = ("x", "n1", "r1", "qkv", "ao", "lse", "h1", "n2", "r2", "gu", "u", "n1T", "aoT", "n2T", "uT",
                 "moe")  # *T: fp8 copies; moe: saved routing / expert buffers


class Backbone:
    """The 12 transformer layers + final norm over a batch of sequences where
    the first ``n_causal`` use the causal mask and the rest the prefix mask."""

    def __init__(self, store: ParamStore, cfg: ModelConfig, fp8=None):
        self.st = store
        self.cfg = cfg
        self.rope = rope_table(cfg.max_seq_len, cfg.head_dim).to(store.device)
        self.fp8 = fp8  # Fp8Recipe: the backbone linears run in fp8 (chessdecoder_b200/fp8.py)
        # MoE variant: with keep_routing set, each forward leaves its per-layer
        # decisions in `routing` as (expert [T, 2] int32, slot [T, 2] int32,
        # -1 = dropped) for inspection (load balance, parity checks)
        self.keep_routing = False
        self.routing = None

    def cast_fp8_weights(self):
        """e4m3 copies (and their transposes) of this step's backbone weights."""
        st, E, F = self.st, self.cfg.embed_dim, self.cfg.ff
        for i in range(self.cfg.num_layers):
            p = f"layers.{i}."
            self.fp8.cast_weights(i, {
                "qkv": st.span(p + "attn.q_proj.weight", p + "attn.v_proj.weight", st.flat).view(3 * E, E),
                "o": st.param(p + "attn.output_proj.weight"),
                "13": st.span(p + "mlp.w1.weight", p + "mlp.w3.weight", st.flat).view(2 * F, E),
                "2": st.param(p + "mlp.w2.weight")})

    # -- MoE MLP (csrc/moe.cu; semantics restated by oracle/moe.py) ------------
    def _moe_fwd(self, i, w, h1, n_seg, T, dev):
        """Router -> top-2 / capacity slots -> per-expert SwiGLU GEMMs on the
        expert-major rows -> weighted combine into the fp32 residual stream.
        The router runs in fp32 (fp32 normalised input and weights) so that the
        discrete top-2 / capacity decisions see fp32 logits."""
        cfg = self.cfg
        E, F, X = cfg.embed_dim, cfg.ff, cfg.moe_experts
        cap = math.ceil(cfg.moe_capacity * 2 * (T // n_seg) / X)
        rows_e = n_seg * cap
        R = X * rows_e
        n2 = torch.empty(T, E, device=dev, dtype=torch.bfloat16)
        n2_32 = torch.empty(T, E, device=dev)
        r2 = torch.empty(T, device=dev)
        K.rmsnorm_fwd(h1, w["s2"], y16=n2, y32=n2_32, rstd=r2)
        logits = torch.empty(T, X, device=dev)
        K.gemm_f32(n2_32, self.st.param(f"layers.{i}.mlp.router.weight"), logits)
        del n2_32
        m = {"n2": n2, "r2": r2, "rows_e": rows_e,
             "expert": torch.empty(T, 2, dtype=torch.int32, device=dev), "weight": torch.empty(T, 2, device=dev),
             "probs": torch.empty(T, X, device=dev), "slot": torch.empty(T, 2, dtype=torch.int32, device=dev)}
        src = torch.empty(R, dtype=torch.int32, device=dev)
        ws = torch.empty(K.moe_route_workspace(T, n_seg, X), dtype=torch.uint8, device=dev)
        K.moe_route(logits, n_seg, cap, m["expert"], m["weight"], m["probs"], m["slot"], src, ws)
        xe = torch.empty(R, E, device=dev, dtype=torch.bfloat16)
        K.moe_dispatch(n2, src, xe)
        gu = torch.empty(R, 2 * F, device=dev, dtype=torch.bfloat16)
        u = torch.empty(R, F, device=dev, dtype=torch.bfloat16)
        ye = torch.empty(R, E, device=dev, dtype=torch.bfloat16)
        for e in range(X):
            r = slice(e * rows_e, (e + 1) * rows_e)
            K.gemm(xe[r], w["w13"][e], kind=K.EPI_SWIGLU, out=u[r], out2=gu[r], half_n=F)
            K.gemm(u[r], w["w2"][e], kind=K.EPI_STORE_BF16, out=ye[r])
        out = torch.empty(T, E, device=dev)
        K.moe_combine(ye, m["slot"], m["weight"], h1, out)
        m.update(xe=xe, gu=gu, u=u, ye=ye)
        return out, m

    def _moe_bwd(self, w, g, m, dh):
        """Gradient of the MoE MLP: returns d(mlp_norm output) [T, E] fp32 and
        accumulates the router / expert weight gradients."""
        cfg = self.cfg
        E, F, X = cfg.embed_dim, cfg.ff, cfg.moe_experts
        T = dh.shape[0]
        dev = dh.device
        rows_e = m["rows_e"]
        R = X * rows_e
        dye = torch.empty(R, E, device=dev, dtype=torch.bfloat16)
        dweight = torch.empty(T, 2, device=dev)
        K.moe_combine_bwd(dh, m["ye"], m["slot"], m["weight"], dye, dweight)
        du = torch.empty(R, F, device=dev, dtype=torch.bfloat16)
        dgu = torch.empty(R, 2 * F, device=dev, dtype=torch.bfloat16)
        dxe = torch.empty(R, E, device=dev, dtype=torch.bfloat16)
        for e in range(X):
            r = slice(e * rows_e, (e + 1) * rows_e)
            K.gemm(dye[r], w["w2"][e], b_mn=True, kind=K.EPI_STORE_BF16, out=du[r])
            K.gemm(dye[r], m["u"][r], a_mn=True, b_mn=True, kind=K.EPI_ATOMIC_F32, out=g["w2"][e])
            K.swiglu_bwd(du[r], m["gu"][r], dgu[r])
            K.gemm(dgu[r], w["w13"][e], b_mn=True, kind=K.EPI_STORE_BF16, out=dxe[r])
            K.gemm(dgu[r], m["xe"][r], a_mn=True, b_mn=True, kind=K.EPI_ATOMIC_F32, out=g["w13"][e])
        ldd = (X + 7) // 8 * 8
        dlog = torch.empty(T, ldd, device=dev, dtype=torch.bfloat16)
        K.moe_route_bwd(m["probs"], m["expert"], dweight, dlog)
        dn = torch.empty(T, E, device=dev)
        K.moe_gather_sum(dxe, m["slot"], dn)
        K.gemm(dlog, w["router"], b_mn=True, kind=K.EPI_ACCUM_F32, out=dn, K=X)
        K.gemm(dlog, m["n2"], a_mn=True, b_mn=True, kind=K.EPI_ATOMIC_F32, out=g["router"], M=X)
        return dn

    def _f8(self, i, lin, a_kind, a_fmt, b_kind, b_fmt):
        f = self.fp8
        return (a_fmt, b_fmt, f.sinv(f.site(i, lin, a_kind)), f.sinv(f.site(i, lin, b_kind)))

    def _w(self, i):
        st, p = self.st, f"layers.{i}."
        wqkv = st.span(p + "attn.q_proj.weight", p + "attn.v_proj.weight").view(3 * self.cfg.embed_dim,
                                                                                 self.cfg.embed_dim)
        d = dict(wqkv=wqkv, wo=st.bf16(p + "attn.output_proj.weight"), s1=st.param(p + "sa_norm.scale"),
                 s2=st.param(p + "mlp_norm.scale"))
        if self.cfg.moe_experts:
            d.update(router=st.bf16(p + "mlp.router.weight"), w13=st.bf16(p + "mlp.experts.w13"),
                     w2=st.bf16(p + "mlp.experts.w2"))
        else:
            d.update(w13=st.span(p + "mlp.w1.weight", p + "mlp.w3.weight").view(2 * self.cfg.ff, self.cfg.embed_dim),
                     w2=st.bf16(p + "mlp.w2.weight"))
        return d

    def _g(self, i):
        st, p = self.st, f"layers.{i}."
        E, F = self.cfg.embed_dim, self.cfg.ff
        gqkv = st.span(p + "attn.q_proj.weight", p + "attn.v_proj.weight", st.grad).view(3 * E, E)
        d = dict(wqkv=gqkv, wo=st.grad_of(p + "attn.output_proj.weight"), s1=st.grad_of(p + "sa_norm.scale"),
                 s2=st.grad_of(p + "mlp_norm.scale"))
        if self.cfg.moe_experts:
            d.update(router=st.grad_of(p + "mlp.router.weight"), w13=st.grad_of(p + "mlp.experts.w13"),
                     w2=st.grad_of(p + "mlp.experts.w2"))
        else:
            d.update(w13=st.span(p + "mlp.w1.weight", p + "mlp.w3.weight", st.grad).view(2 * F, E),
                     w2=st.grad_of(p + "mlp.w2.weight"))
        return d

    def forward(self, h, nseq, n_causal, S, bid32=None, meta=None, want_f32=False, rope=None):
        """rope: optional [S, head_dim/2, 2] table whose row s rotates sequence
        position s (the module's ``input_pos``: table = cache[input_pos]);
        default the cache itself (position s = s)."""
        cfg = self.cfg
        rope = self.rope if rope is None else rope
        E, F, H = cfg.embed_dim, cfg.ff, cfg.num_heads
        T = h.shape[0]
        dev = h.device
        saved = []
        x = h
        f8 = self.fp8
        E4, E5 = K.FP8_E4M3, K.FP8_E5M2
        # MoE capacity is per forward pass: the merged batch routes its two halves separately
        n_seg = 2 if 0 < n_causal < nseq and 2 * n_causal == nseq else 1
        for i in range(cfg.num_layers):
            w = self._w(i)
            s = LayerSaved()
            s.x = x
            s.r1 = torch.empty(T, device=dev)
            # fp8 after the first step: the norm writes the e4m3 GEMM input itself
            fq = f8.fused(f8.site(i, "qkv", "x"), E4, T, E) if f8 is not None else None
            if fq is not None:
                s.n1, s.n1T = None, fq[0]
                K.rmsnorm_fwd(x, w["s1"], rstd=s.r1, q8=fq[1])
            else:
                s.n1 = torch.empty(T, E, device=dev, dtype=torch.bfloat16)
                K.rmsnorm_fwd(x, w["s1"], y16=s.n1, rstd=s.r1)
            s.qkv = torch.empty(T, 3 * E, device=dev, dtype=torch.bfloat16)
            if f8 is None:
                K.gemm(s.n1, w["wqkv"], kind=K.EPI_ROPE_BF16, out=s.qkv, rope=rope, seq_len=S, rope_cols=2 * E)
            else:
                if fq is None:
                    s.n1T = f8.cast(s.n1, f8.site(i, "qkv", "x"), E4)
                    s.n1 = None
                K.gemm(s.n1T, f8.weights[(i, "qkv")], kind=K.EPI_ROPE_BF16, out=s.qkv, rope=rope, seq_len=S,
                       rope_cols=2 * E, fp8=self._f8(i, "qkv", "x", E4, "w", E4))
            s.ao = torch.empty(T, E, device=dev, dtype=torch.bfloat16)
            s.lse = torch.empty(nseq * H * S, device=dev)
            K.attn_fwd(s.qkv, s.ao, s.lse, nseq, n_causal, S, H, bid32, meta)
            s.h1 = torch.empty(T, E, device=dev)
            if f8 is None:
                K.gemm(s.ao, w["wo"], kind=K.EPI_RESID_F32, out=s.h1, resid=x)
            else:
                a8 = s.aoT = f8.cast(s.ao, f8.site(i, "o", "x"), E4)
                K.gemm(a8, f8.weights[(i, "o")], kind=K.EPI_RESID_F32, out=s.h1, resid=x,
                       fp8=self._f8(i, "o", "x", E4, "w", E4))
            if cfg.moe_experts:
                out, s.moe = self._moe_fwd(i, w, s.h1, n_seg, T, dev)
                s.n2, s.r2 = s.moe["n2"], s.moe["r2"]
                saved.append(s)
                x = out
                continue
            s.r2 = torch.empty(T, device=dev)
            fq = f8.fused(f8.site(i, "13", "x"), E4, T, E) if f8 is not None else None
            if fq is not None:
                s.n2, s.n2T = None, fq[0]
                K.rmsnorm_fwd(s.h1, w["s2"], rstd=s.r2, q8=fq[1])
            else:
                s.n2 = torch.empty(T, E, device=dev, dtype=torch.bfloat16)
                K.rmsnorm_fwd(s.h1, w["s2"], y16=s.n2, rstd=s.r2)
            s.gu = torch.empty(T, 2 * F, device=dev, dtype=torch.bfloat16)
            s.u = torch.empty(T, F, device=dev, dtype=torch.bfloat16)
            out = torch.empty(T, E, device=dev)
            if f8 is None:
                K.gemm(s.n2, w["w13"], kind=K.EPI_SWIGLU, out=s.u, out2=s.gu, half_n=F)
                K.gemm(s.u, w["w2"], kind=K.EPI_RESID_F32, out=out, resid=s.h1)
            else:
                if fq is None:
                    s.n2T = f8.cast(s.n2, f8.site(i, "13", "x"), E4)
                    s.n2 = None
                K.gemm(s.n2T, f8.weights[(i, "13")], kind=K.EPI_SWIGLU, out=s.u, out2=s.gu, half_n=F,
                       fp8=self._f8(i, "13", "x", E4, "w", E4))
                u8 = s.uT = f8.cast(s.u, f8.site(i, "2", "x"), E4)
                s.u = None
                K.gemm(u8, f8.weights[(i, "2")], kind=K.EPI_RESID_F32, out=out, resid=s.h1,
                       fp8=self._f8(i, "2", "x", E4, "w", E4))
            saved.append(s)
            x = out
        if cfg.moe_experts and self.keep_routing:
            self.routing = [(s.moe["expert"], s.moe["slot"]) for s in saved]
        hN16 = torch.empty(T, E, device=dev, dtype=torch.bfloat16)
        hN32 = torch.empty(T, E, device=dev) if want_f32 else None
        rN = torch.empty(T, device=dev)
        K.rmsnorm_fwd(x, self.st.param("norm.scale"), y16=hN16, y32=hN32, rstd=rN)
        return hN16, hN32, (saved, x, rN, nseq, n_causal, S, bid32, meta, rope)

    def backward(self, dhN, ctx, on_layer_done: Optional[Callable[[int], None]] = None):
        """dhN: f32 [T,E] gradient of the final-norm output.  Accumulates every
        backbone weight gradient into the store; returns d(embedding output)."""
        saved, xL, rN, nseq, n_causal, S, bid32, meta, rope = ctx
        cfg, st = self.cfg, self.st
        E, F, H = cfg.embed_dim, cfg.ff, cfg.num_heads
        T = dhN.shape[0]
        dev = dhN.device
        dh = torch.empty(T, E, device=dev)
        dh16 = torch.empty(T, E, device=dev, dtype=torch.bfloat16)
        f8 = self.fp8
        E4, E5 = K.FP8_E4M3, K.FP8_E5M2
        # fp8 after the first step: each norm backward writes the e5m2 dY of the
        # linear below it (w2's from the final norm and from each sa_norm, the
        # output projection's from each mlp_norm) and the SwiGLU backward that of
        # w1|w3
        fq = f8.fused(f8.site(cfg.num_layers - 1, "2", "g"), E5, T, E) if f8 is not None else None
        g2_8 = fq[0] if fq is not None else None
        K.rmsnorm_bwd(dhN, xL, st.param("norm.scale"), rN, dx=dh, dx16=None if fq else dh16,
                      dscale=st.grad_of("norm.scale"), q8=fq[1] if fq else None)
        if on_layer_done is not None:
            on_layer_done(cfg.num_layers)  # heads + final norm done
        dgu = torch.empty(T, 2 * F, device=dev, dtype=torch.bfloat16)
        du = torch.empty(T, F, device=dev, dtype=torch.bfloat16)
        dn = torch.empty(T, E, device=dev, dtype=torch.bfloat16)
        dh1 = torch.empty(T, E, device=dev)
        dh1_16 = torch.empty(T, E, device=dev, dtype=torch.bfloat16)
        dao = torch.empty(T, E, device=dev, dtype=torch.bfloat16)
        dqkv = torch.empty(T, 3 * E, device=dev, dtype=torch.bfloat16)
        dsum = torch.empty(nseq * H * S, device=dev)
        for i in reversed(range(cfg.num_layers)):
            s = saved[i]
            w, g = self._w(i), self._g(i)
            if cfg.moe_experts:
                dn_moe = self._moe_bwd(w, g, s.moe, dh)
                K.rmsnorm_bwd(dn_moe, s.h1, w["s2"], s.r2, dx=dh1, dx16=dh1_16, dscale=g["s2"], dres=dh)
            elif f8 is None:
                # MLP block: [dg | du] = SwiGLU backward of dh W2, fused into that GEMM's (TMA-fed) epilogue
                K.gemm(dh16, w["w2"], b_mn=True, kind=K.EPI_DSWIGLU, out=dgu, aux=s.gu, half_n=F, N=F)
                K.gemm(dh16, s.u, a_mn=True, b_mn=True, kind=K.EPI_ATOMIC_F32, out=g["w2"])
                K.gemm(dgu, w["w13"], b_mn=True, kind=K.EPI_STORE_BF16, out=dn)
                K.gemm(dgu, s.n2, a_mn=True, b_mn=True, kind=K.EPI_ATOMIC_F32, out=g["w13"])
            else:
                g8 = g2_8 if g2_8 is not None else f8.cast(dh16, f8.site(i, "2", "g"), E5)
                K.gemm(g8, f8.weights[(i, "2")], b_mn=True, kind=K.EPI_STORE_BF16, out=du,
                       fp8=self._f8(i, "2", "g", E5, "w", E4))
                fq = f8.fused(f8.site(i, "13", "g"), E5, T, 2 * F)
                if fq is not None:
                    K.swiglu_bwd(du, s.gu, q8=fq[1])
                else:
                    K.swiglu_bwd(du, s.gu, dgu)
                K.gemm(g8, s.uT, a_mn=True, b_mn=True, kind=K.EPI_ATOMIC_F32, out=g["w2"],
                       fp8=self._f8(i, "2", "g", E5, "x", E4))
                g8 = fq[0] if fq is not None else f8.cast(dgu, f8.site(i, "13", "g"), E5)
                K.gemm(g8, f8.weights[(i, "13")], b_mn=True, kind=K.EPI_STORE_BF16, out=dn,
                       fp8=self._f8(i, "13", "g", E5, "w", E4))
                K.gemm(g8, s.n2T, a_mn=True, b_mn=True, kind=K.EPI_ATOMIC_F32, out=g["w13"],
                       fp8=self._f8(i, "13", "g", E5, "x", E4))
            go_8 = None
            if not cfg.moe_experts:
                fq = f8.fused(f8.site(i, "o", "g"), E5, T, E) if f8 is not None else None
                go_8 = fq[0] if fq is not None else None
                K.rmsnorm_bwd(dn, s.h1, w["s2"], s.r2, dx=dh1, dx16=None if fq else dh1_16, dscale=g["s2"], dres=dh,
                              q8=fq[1] if fq else None)
            if on_layer_done is not None:
                on_layer_done(("mlp", i))  # the MLP block's gradients (and its norm's) are final
            # attention block
            if f8 is None:
                K.gemm(dh1_16, w["wo"], b_mn=True, kind=K.EPI_STORE_BF16, out=dao)
                K.gemm(dh1_16, s.ao, a_mn=True, b_mn=True, kind=K.EPI_ATOMIC_F32, out=g["wo"])
            else:
                g8 = go_8 if go_8 is not None else f8.cast(dh1_16, f8.site(i, "o", "g"), E5)
                K.gemm(g8, f8.weights[(i, "o")], b_mn=True, kind=K.EPI_STORE_BF16, out=dao,
                       fp8=self._f8(i, "o", "g", E5, "w", E4))
                K.gemm(g8, s.aoT, a_mn=True, b_mn=True, kind=K.EPI_ATOMIC_F32, out=g["wo"],
                       fp8=self._f8(i, "o", "g", E5, "x", E4))
            fq = f8.fused(f8.site(i, "qkv", "g"), E5, T, 3 * E) if f8 is not None else None
            if fq is not None and K.attn_bwd_q8(s.qkv, s.ao, dao, s.lse, dsum, fq[1], nseq, n_causal, S, H, bid32,
                                               meta, rope=rope):
                gqkv8 = fq[0]  # the attention backward wrote the e5m2 dY of the q|k|v projection itself
            else:
                gqkv8 = None
                K.attn_bwd(s.qkv, s.ao, dao, s.lse, dsum, dqkv, nseq, n_causal, S, H, bid32, meta, rope=rope)
            if f8 is None:
                K.gemm(dqkv, w["wqkv"], b_mn=True, kind=K.EPI_STORE_BF16, out=dn)
                K.gemm(dqkv, s.n1, a_mn=True, b_mn=True, kind=K.EPI_ATOMIC_F32, out=g["wqkv"])
            else:
                g8 = gqkv8 if gqkv8 is not None else f8.cast(dqkv, f8.site(i, "qkv", "g"), E5)
                K.gemm(g8, f8.weights[(i, "qkv")], b_mn=True, kind=K.EPI_STORE_BF16, out=dn,
                       fp8=self._f8(i, "qkv", "g", E5, "w", E4))
                K.gemm(g8, s.n1T, a_mn=True, b_mn=True, kind=K.EPI_ATOMIC_F32, out=g["wqkv"],
                       fp8=self._f8(i, "qkv", "g", E5, "x", E4))
            fq = f8.fused(f8.site(i - 1, "2", "g"), E5, T, E) if (f8 is not None and i > 0) else None
            g2_8 = fq[0] if fq is not None else None
            K.rmsnorm_bwd(dn, s.x, w["s1"], s.r1, dx=dh, dx16=None if fq else dh16, dscale=g["s1"], dres=dh1,
                          q8=fq[1] if fq else None)
            if on_layer_done is not None:
                on_layer_done(i)
        return dh


# ---------------------------------------------------------------------------
# Embedding + Fourier front end
# ---------------------------------------------------------------------------
class FrontEnd:
    def __init__(self, store: ParamStore, cfg: ModelConfig):
        self.st = store
        self.cfg = cfg
        self.wl_c = make_wl_buckets(cfg.n_buckets, cfg.wl_sigma).to(store.device)
        self.d_c = make_d_buckets(cfg.n_buckets).to(store.device)

    def forward(self, db: DeviceBatch, n_copies: int, snap: bool = True):
        """snap=False: the placeholder values are used as given (the module
        forward, whose caller snapped them with prepare_fourier_inputs)."""
        cfg, st = self.cfg, self.st
        E, nf = cfg.embed_dim, cfg.num_fourier_freq
        dev = db.ids.device
        Nf = db.frows.numel()
        fvals = torch.empty(max(Nf, 1), device=dev)
        feat = torch.empty(max(Nf, 1), 2 * nf, device=dev)
        frows_out = torch.empty(max(Nf, 1), E, device=dev)
        if Nf:
            K.fourier_features(db.wl_t, db.d_t, db.wl_pos, db.d_pos, self.wl_c if snap else None,
                               self.d_c if snap else None,
                               st.param("fourier_encoder.frequencies"), db.frows, fvals, feat)
            K.gemm_f32(feat, st.param("fourier_encoder.proj.weight"), frows_out,
                       bias=st.param("fourier_encoder.proj.bias"), M=Nf)
        h0 = torch.empty(n_copies * db.ids.numel(), E, device=dev)
        K.embed_fwd(db.ids, st.param("tok_embedding.weight"), db.slot, frows_out, h0, n_copies=n_copies)
        return h0, (fvals, feat, Nf)

    def backward(self, db: DeviceBatch, dh0, ctx, n_copies: int):
        fvals, feat, Nf = ctx
        st, cfg = self.st, self.cfg
        E = cfg.embed_dim
        dev = dh0.device
        dfr = torch.empty(max(Nf, 1), E, device=dev)
        K.embed_bwd(db.ids, dh0, db.slot, st.grad_of("tok_embedding.weight"), dfr, n_copies=n_copies)
        if Nf:
            # d proj.weight [E, 2F] += dfr^T feat ; d proj.bias += colsum(dfr) ; dfeat = dfr W
            K.gemm_f32(dfr, feat, st.grad_of("fourier_encoder.proj.weight"), a_t=True, b_t=True, accumulate=True,
                       M=E, N=feat.shape[1], K=Nf)
            ones = torch.ones(1, Nf, device=dev)
            K.gemm_f32(ones, dfr, st.grad_of("fourier_encoder.proj.bias").view(1, E), b_t=True, accumulate=True,
                       M=1, N=E, K=Nf)
            dfeat = torch.empty(Nf, feat.shape[1], device=dev)
            K.gemm_f32(dfr, st.param("fourier_encoder.proj.weight"), dfeat, b_t=True, M=Nf, N=feat.shape[1], K=E)
            K.fourier_bwd(fvals[:Nf], st.param("fourier_encoder.frequencies"), dfeat,
                          st.grad_of("fourier_encoder.frequencies"))


# ---------------------------------------------------------------------------
# Heads + losses (forward and backward in one pass over the gathered rows)
# ---------------------------------------------------------------------------
class Heads:
    """Board head on pass-1 rows, policy head on move rows, WL / D value heads,
    each with its loss and its gradient; accumulates dL/dhN."""

    def __init__(self, store: ParamStore, cfg: ModelConfig, loss_weights=(5.0, 1.0, 1.0, 1.0), fp8=None):
        self.st = store
        self.cfg = cfg
        self.fp8 = fp8  # Fp8Recipe with head sites: the head linears run on fp8 GEMMs
        self.w_move, self.w_board, self.w_wl, self.w_d = loss_weights[:4]
        self.w_think = loss_weights[4] if len(loss_weights) > 4 else 0.0
        if self.w_think and not cfg.finetune:
            raise ValueError("a thinking-move loss weight needs ModelConfig(finetune=True)")
        self.wl_c = make_wl_buckets(cfg.n_buckets, cfg.wl_sigma).to(store.device)
        self.d_c = make_d_buckets(cfg.n_buckets).to(store.device)

    def run(self, db: DeviceBatch, hN16, losses, metrics=None):
        """losses: f32 [5] (move, board, wl, d, thinking move), accumulated.  Returns dhN f32 [2*B*S, E]."""
        st, cfg = self.st, self.cfg
        E = cfg.embed_dim
        BS = db.B * db.S
        dev = hN16.device
        T = hN16.shape[0]
        dhN = torch.empty(T, E, device=dev)
        dhN[BS:].zero_()
        norms = db.norms
        # fp8: the pass-1 and pass-2 rows quantised once each (the board head reads
        # the former, the policy / thinking heads gather from the latter)
        self._h8 = None
        if self.fp8 is not None:
            from .fp8 import _empty8
            f = self.fp8
            self._h8 = _empty8(T, E, torch.float8_e4m3fn, dev)
            f.cast(hN16[:BS], f.head_site("h_causal", "x"), K.FP8_E4M3, out=self._h8[:BS])
            f.cast(hN16[BS:], f.head_site("h_prefix", "x"), K.FP8_E4M3, out=self._h8[BS:])
        # ---- board head over pass-1 rows -----------------------------------
        nbv = V.board_vocab_size
        logits = torch.empty(BS, 44, device=dev)
        xc8 = self._h8[:BS] if self._h8 is not None else None
        self._lin_fwd("board_head", hN16[:BS], xc8, "h_causal", logits, N=nbv)
        dl = torch.empty(BS, 48, device=dev, dtype=torch.bfloat16)
        bam = metrics.get("board_argmax") if metrics is not None else None
        K.softmax_ce(logits, db.board_t, db.board_w, norms[1:2], self.w_board, dlogits=dl,
                     dbias=st.grad_of("board_head.bias"), loss_out=losses[1:2], argmax=bam, ncls=nbv)
        self._lin_bwd("board_head", dl, nbv, hN16[:BS], xc8, "h_causal", dhN[:BS])
        # ---- policy head over gathered move rows; thinking head (finetune) ----
        pam = metrics.get("move_argmax") if metrics is not None else None
        self._move_head("policy_head", db.prow, db.pt, norms[0:1], self.w_move, hN16, dhN, losses[0:1], pam)
        if db.trow is not None and db.trow.numel():
            tam = metrics.get("thinking_argmax") if metrics is not None else None
            self._move_head("thinking_policy_head", db.trow, db.tt, norms[4:5], self.w_think, hN16, dhN,
                            losses[4:5], tam)
        # ---- value heads ------------------------------------------------------
        self._value("wl_head", db.wrow, db.wtgt, db.wvalid, self.wl_c, norms[2:3], self.w_wl, hN16, dhN,
                    losses[2:3])
        self._value("d_head", db.drow, db.dtgt, db.dvalid, self.d_c, norms[3:4], self.w_d, hN16, dhN, losses[3:4])
        return dhN

    def _move_head(self, name, rows, tgt, norm, weight, hN16, dhN, loss, argmax=None):
        """Move-vocabulary head + masked CE on gathered rows (train.py:204-207;
        the thinking head of chessdecoder/finetune/train.py:315-318 is the
        same statement)."""
        n = rows.numel()
        if n == 0:
            return
        st, E, dev = self.st, self.cfg.embed_dim, hN16.device
        nmv = V.move_vocab_size
        hp, hp8 = None, None
        if self._h8 is None:
            hp = torch.empty(n, E, device=dev, dtype=torch.bfloat16)
            K.gather_rows_bf16(hN16, rows, hp)
        else:  # gather the 8-bit rows (E bytes = E / 2 bf16-sized elements)
            from .fp8 import _empty8
            hp8 = _empty8(n, E, torch.float8_e4m3fn, dev)
            K.gather_rows_bf16(self._h8.view(torch.bfloat16), rows, hp8.view(torch.bfloat16))
        lp = torch.empty(n, nmv, device=dev)
        self._lin_fwd(name, hp, hp8, "h_prefix", lp)
        dlp = torch.empty(n, 1928, device=dev, dtype=torch.bfloat16)
        K.softmax_ce(lp, tgt, None, norm, weight, dlogits=dlp, dbias=st.grad_of(f"{name}.bias"), loss_out=loss,
                     argmax=argmax, ncls=nmv)
        dhp = torch.empty(n, E, device=dev)
        self._lin_bwd(name, dlp, nmv, hp, hp8, "h_prefix", dhp)
        K.scatter_add_rows(dhp, rows, dhN)

    def _value(self, name, rows, tgt, valid, centers, norm, weight, hN16, dhN, loss):
        n = rows.numel()
        if n == 0:
            return
        st, cfg = self.st, self.cfg
        E, hv, nb = cfg.embed_dim, cfg.value_hidden_size, cfg.n_buckets
        dev = hN16.device
        x = torch.empty(n, E, device=dev, dtype=torch.bfloat16)
        K.gather_rows_bf16(hN16, rows, x)
        z1 = torch.empty(n, hv, device=dev)
        lin0 = f"{name}.mlp.0"
        x8 = None
        if self.fp8 is not None:
            x8 = self.fp8.cast(x, self.fp8.head_site(lin0, "x"), K.FP8_E4M3)
        self._lin_fwd(lin0, x, x8, lin0, z1)
        act = torch.empty(n, hv, device=dev)
        dlog = torch.empty(n, nb, device=dev)
        dz = torch.empty(n, hv, device=dev, dtype=torch.bfloat16)
        K.value_tail(z1, st.param(f"{name}.mlp.2.weight"), st.param(f"{name}.mlp.2.bias"), tgt, valid, centers, norm,
                     weight, act, dlog, dz, db1=st.grad_of(f"{name}.mlp.0.bias"), loss_out=loss)
        # second Linear: dW2 += dlog^T act, db2 += colsum(dlog)
        K.gemm_f32(dlog, act, st.grad_of(f"{name}.mlp.2.weight"), a_t=True, b_t=True, accumulate=True, M=nb, N=hv, K=n)
        ones = torch.ones(1, n, device=dev)
        K.gemm_f32(ones, dlog, st.grad_of(f"{name}.mlp.2.bias").view(1, nb), b_t=True, accumulate=True, M=1, N=nb,
                   K=n)
        # first Linear: dX = dz W1, dW1 += dz^T X
        dx = torch.empty(n, E, device=dev)
        self._lin_bwd(lin0, dz, hv, x, x8, lin0, dx)
        K.scatter_add_rows(dx, rows, dhN)

    # ---- head linears: bf16 GEMMs, or the fp8 recipe's e4m3 / e5m2 GEMMs -------
    def _lin_fwd(self, name, x16, x8, xsite, out, N=None):
        """out (fp32) = x W^T + b."""
        st, f = self.st, self.fp8
        if f is None:
            K.gemm(x16, st.bf16(f"{name}.weight"), kind=K.EPI_STORE_F32, out=out, bias=st.param(f"{name}.bias"), N=N)
            return
        K.gemm(x8, f.weights[("head", name)], kind=K.EPI_STORE_F32, out=out, bias=st.param(f"{name}.bias"), N=N,
               fp8=(K.FP8_E4M3, K.FP8_E4M3, f.sinv(f.head_site(xsite, "x")), f.sinv(f.head_site(name, "w"))))

    def _lin_bwd(self, name, g16, ncols, x16, x8, xsite, dx):
        """dx (fp32) = g W and dW += g^T x for the bf16 logit gradient g [rows, >= ncols]."""
        st, f = self.st, self.fp8
        n = g16.shape[0]
        gw = st.grad_of(f"{name}.weight")
        if f is None:
            K.gemm(g16, st.bf16(f"{name}.weight"), b_mn=True, kind=K.EPI_STORE_F32, out=dx, K=ncols)
            K.gemm(g16, x16, a_mn=True, b_mn=True, kind=K.EPI_ATOMIC_F32, out=gw, M=ncols, K=n)
            return
        gs, ws, xs = f.head_site(name, "g"), f.head_site(name, "w"), f.head_site(xsite, "x")
        g8 = f.cast(g16[:, :ncols], gs, K.FP8_E5M2)
        K.gemm(g8, f.weights[("head", name)], b_mn=True, kind=K.EPI_STORE_F32, out=dx, K=ncols,
               fp8=(K.FP8_E5M2, K.FP8_E4M3, f.sinv(gs), f.sinv(ws)))
        K.gemm(g8, x8, a_mn=True, b_mn=True, kind=K.EPI_ATOMIC_F32, out=gw, M=ncols, K=n,
               fp8=(K.FP8_E5M2, K.FP8_E4M3, f.sinv(gs), f.sinv(xs)))

    def head_linears(self):
        names = ["board_head", "policy_head", "wl_head.mlp.0", "d_head.mlp.0"]
        return names + (["thinking_policy_head"] if self.cfg.finetune else [])

    def cast_fp8_weights(self):
        f = self.fp8
        for name in self.head_linears():
            f.weights[("head", name)] = f.cast(self.st.param(f"{name}.weight"), f.head_site(name, "w"), K.FP8_E4M3)


# ---------------------------------------------------------------------------
# The training step
# ---------------------------------------------------------------------------
def pipelined_steps(step_fn, batches, metrics=None):
    """Runs step_fn(batch, metrics) -> device losses over `batches`, keeping
    one step in flight: each step's losses are copied to pinned host memory
    behind its kernels and read after the next step has been enqueued, so the
    host's batch preparation and launches overlap the device's work.  Yields
    (i, host losses) in order; every step's losses are read."""
    pending = None
    for i, b in enumerate(batches):
        losses = step_fn(b, metrics)
        host = torch.empty(losses.shape, dtype=losses.dtype, pin_memory=losses.is_cuda)
        host.copy_(losses, non_blocking=True)
        ev = None
        if losses.is_cuda:
            ev = torch.cuda.Event()
            ev.record()
        if pending is not None:
            if pending[2] is not None:
                pending[2].synchronize()
            yield pending[0], pending[1]
        pending = (i, host, ev)
    if pending is not None:
        if pending[2] is not None:
            pending[2].synchronize()
        yield pending[0], pending[1]


class TrainStep:
    """One optimizer step of ChessDecoder pretraining on B200.

    ``step(batch)`` = prepare_batch + forward_backward + (all-reduce) +
    clip + AdamW.  ``grad_hook(layer_index)`` (optional) is called as soon as
    the gradients of a layer are final; the data-parallel wrapper uses it to
    start bucket all-reduces during the backward.
    """

    def __init__(self, cfg: ModelConfig, device="cuda", seed=0, lr=3e-4, weight_decay=0.1, betas=(0.9, 0.999),
                 eps=1e-8, max_norm=10.0, loss_weights=(5.0, 1.0, 1.0, 1.0), state_dict=None, fp8: bool = False):
        self.cfg = cfg
        self.device = torch.device(device)
        self.store = ParamStore(cfg, self.device)
        sd = state_dict if state_dict is not None else init_reference_weights(cfg, seed)
        self.store.load_state_dict({k: v.to(self.device) for k, v in sd.items()})
        self.fp8 = None
        if fp8 and cfg.moe_experts:
            raise ValueError("the fp8 recipe covers the dense MLP only; the MoE variant runs in bf16")
        if fp8:
            from .fp8 import Fp8Recipe
            heads = ["board_head", "policy_head", "wl_head.mlp.0", "d_head.mlp.0"]
            self.fp8 = Fp8Recipe(cfg.num_layers, self.device,
                                 heads=heads + (["thinking_policy_head"] if cfg.finetune else []))
        self.backbone = Backbone(self.store, cfg, self.fp8)
        self.front = FrontEnd(self.store, cfg)
        self.heads = Heads(self.store, cfg, loss_weights, fp8=self.fp8)
        self.lr, self.wd, self.betas, self.eps, self.max_norm = lr, weight_decay, betas, eps, max_norm
        self.grad_hook: Optional[Callable[[int], None]] = None
        self.grad_scale = 1.0
        self.partial = torch.empty(1024, device=self.device)
        self.loss_weights = loss_weights
        self.grad_accum = 1  # micro-batches per optimizer step (config.yaml gradient_accumulation_steps)

    def forward_backward(self, db: DeviceBatch, metrics=None, zero_grad: bool = True, sync: bool = True):
        """Loss forward + full backward into store.grad.  Returns losses f32
        [5] = (move, board, wl, d, thinking move) on the device (the last is 0
        outside the finetune step).  zero_grad=False accumulates onto the
        gradients of earlier micro-batches (gradient accumulation,
        chessdecoder/train/train.py:244-250); sync=False skips the
        ``grad_hook`` (the data-parallel all-reduce runs during the last
        micro-batch only, as average_gradients runs once per optimizer step)."""
        st = self.store
        if zero_grad:
            st.grad.zero_()
        B, S = db.B, db.S
        losses = torch.zeros(5, device=self.device)
        meta = K.attn_meta(db.bid, S)
        if self.fp8 is not None:
            self.backbone.cast_fp8_weights()
            self.heads.cast_fp8_weights()
        h0, fctx = self.front.forward(db, n_copies=2)
        hN16, _, bctx = self.backbone.forward(h0, 2 * B, B, S, db.bid, meta)
        dhN = self.heads.run(db, hN16, losses, metrics)
        hook = self.grad_hook if sync else None
        dh0 = self.backbone.backward(dhN, bctx, hook)
        self.front.backward(db, dh0, fctx, n_copies=2)
        if self.fp8 is not None:
            self.fp8.end_step()
        if hook is not None:
            hook(-1)
        return losses

    def optimizer_step(self, accum: int = 1):
        """Clip + AdamW on the summed gradients of ``accum`` micro-batches:
        the gradients are scaled by 1 / accum (the reference divides each
        micro-batch's loss, train.py:244) and the data-parallel mean, and the
        clip norm is taken on the scaled sum, as clip_grad_norm_ runs after the
        accumulation (train.py:249-250)."""
        st = self.store
        st.step += 1
        K.sumsq(st.grad, self.partial)
        K.adamw(st.flat, st.grad, st.exp_avg, st.exp_avg_sq, st.flat16, self.partial, max_norm=self.max_norm,
                lr=self.lr, beta1=self.betas[0], beta2=self.betas[1], eps=self.eps, wd=self.wd, step=st.step,
                grad_scale=self.grad_scale / accum)

    def step(self, batch: dict, metrics=None):
        db = prepare_batch(batch, self.device)
        losses = self.forward_backward(db, metrics)
        self.optimizer_step()
        return losses

    def run(self, batches, metrics=None):
        """Training loop over host batches: yields (i, losses f32 [5] on the
        host) for every batch, one step behind the device — batch i+1 is
        prepared and its step enqueued while step i runs, then step i's losses
        (copied into pinned memory at the end of its step) are read.  The
        reference's loop overlaps the same way: its DataLoader workers build
        the next batch and it reads losses only every log_every_n_steps
        (train/train.py:150, 327)."""
        return pipelined_steps(self.step, batches, metrics)

    def step_accumulated(self, batches, metrics=None):
        """One optimizer step over micro-batches (gradient_accumulation_steps
        = len(batches), train/config.yaml:25); returns each micro-batch's
        losses f32 [5]."""
        out = []
        n = len(batches)
        for i, b in enumerate(batches):
            db = prepare_batch(b, self.device)
            out.append(self.forward_backward(db, metrics, zero_grad=i == 0, sync=i == n - 1))
        self.optimizer_step(accum=n)
        return out

    # -- checkpoints (chessdecoder/utils/training.py:136-157, train/train.py:81-104) --
    def optimizer_state_dict(self) -> dict:
        return self.store.optimizer_state_dict(self.lr, self.betas, self.eps, self.wd)

    def load_optimizer_state_dict(self, sd: dict):
        """AdamW moments and step from a state_dict in the reference layout; the
        configured learning rate is kept (train.py:95-96 re-applies it on resume)."""
        g = self.store.load_optimizer_state_dict(sd)
        self.betas, self.eps, self.wd = tuple(g["betas"]), g["eps"], g["weight_decay"]

    def checkpoint(self, step: int, extra_state: Optional[dict] = None) -> dict:
        """The dict save_training_checkpoint writes: step, model / optimizer /
        scaler state (the bf16 step needs no loss scaling: an empty scaler
        state, as a disabled GradScaler's), plus ``extra_state``."""
        ck = {"step": step, "model_state_dict": self.store.state_dict(),
              "optimizer_state_dict": self.optimizer_state_dict(), "scaler_state_dict": {}}
        if extra_state:
            ck.update(extra_state)
        return ck

    def load_checkpoint(self, ck: dict):
        """Weights and optimizer state from a checkpoint dict (the reference's
        or ``checkpoint()``'s); returns its step."""
        self.store.load_state_dict({k: v.to(self.device) for k, v in ck["model_state_dict"].items()})
        self.load_optimizer_state_dict(ck["optimizer_state_dict"])
        return ck.get("step", 0)

    @staticmethod
    def total(losses, weights=(5.0, 1.0, 1.0, 1.0)):
        return sum(w * losses[i] for i, w in enumerate(weights))


# Loss weights of chessdecoder/finetune/config.yaml (final move, board, wl, d, thinking move).
FINETUNE_LOSS_WEIGHTS = (3.0, 1.0, 3.0, 3.0, 3.0)
