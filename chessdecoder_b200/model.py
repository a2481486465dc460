"""Drop-in ``ChessDecoder`` module: the constructor, attribute tree,
``state_dict`` keys, initial weights and ``forward`` contract of
chessdecoder/models/model.py:55-194, with the forward and backward running on
the chessdecoder_b200 CUDA kernels.

A training loop written against the reference (chessdecoder/train/train.py:
157-253) runs unchanged: ``model(ids, mask_type=..., ...)`` returns the final
hidden states ``h`` [B, S, E] (fp32); ``model.board_head(h)``,
``model.policy_head(h)``, ``model.wl_head(rows)`` and ``model.d_head(rows)``
are callable modules; ``loss.backward()`` (also through ``GradScaler``) fills
``p.grad`` for every parameter; any ``torch.optim`` optimizer updates them.

How it maps onto the kernels:

* On the first CUDA forward every parameter of the flat layout (all but the
  thinking head) is moved into one flat fp32 buffer and the Parameter objects
  are re-pointed at views of it (``p.data``), so optimizers created before or
  after keep working.  A bf16 shadow of the flat buffer feeds the GEMMs; it is
  re-cast whenever a parameter's version counter moved (an optimizer step, a
  ``load_state_dict``).
* The backbone (embedding + Fourier injection, all layers, final norm) is ONE
  autograd node.  Its backward accumulates into one flat fp32 gradient buffer
  whose per-parameter views are the parameters' ``.grad`` (allocated by the
  first backward after ``zero_grad(set_to_none=True)``, reused by the next
  ones), so the backbone gradients are contiguous and ``average_gradients``
  reduces them as a few large buckets in place.
* The heads' ``nn.Linear`` layers are ``Linear`` below: bf16 tcgen05 GEMMs
  with fp32 outputs and fp32 gradients.

The submodules that only hold weights (attention, feed-forward, norms, the
Fourier encoder) run inside ``ChessDecoder.forward``; called on their own they
raise.  CPU tensors raise too: there is no CPU path.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn

from . import kernels as K
from . import ops as _ops  # noqa: F401  (registers the cdk:: custom ops)
from . import vocab as V
from .engine import (Backbone, FrontEnd, ModelConfig, ParamStore, make_d_buckets, make_wl_buckets,
                     rope_table)

_HEADS = ("board_head.", "policy_head.", "wl_head.", "d_head.")


def _cuda_only(what: str):
    raise RuntimeError(f"chessdecoder_b200: {what} runs on CUDA tensors only (no CPU path)")


class _WeightsOnly(nn.Module):
    """A container whose arithmetic runs inside ChessDecoder.forward."""

    def forward(self, *args, **kwargs):
        raise RuntimeError(f"chessdecoder_b200: {type(self).__name__} runs inside ChessDecoder.forward only")


class RMSNorm(_WeightsOnly):
    """torchtune RMSNorm (eps 1e-6, fp32 statistics): parameter ``scale``."""

    def __init__(self, dim: int, eps: float = 1e-6):
        super().__init__()
        self.eps = eps
        self.scale = nn.Parameter(torch.ones(dim))


class RotaryPositionalEmbeddings(_WeightsOnly):
    """Interleaved RoPE, base 10000, cache [max_seq_len, dim/2, 2] (non-persistent
    buffer, so it is not part of the state dict)."""

    def __init__(self, dim: int, max_seq_len: int = 4096, base: int = 10_000):
        super().__init__()
        self.dim, self.max_seq_len, self.base = dim, max_seq_len, base
        self.register_buffer("cache", rope_table(max_seq_len, dim, float(base)), persistent=False)


class MultiHeadAttention(_WeightsOnly):
    def __init__(self, embed_dim, num_heads, num_kv_heads, head_dim, q_proj, k_proj, v_proj, output_proj,
                 pos_embeddings=None, max_seq_len=4096, is_causal=True):
        super().__init__()
        if num_kv_heads != num_heads:
            raise ValueError("grouped-query attention is not part of ChessDecoder")
        self.embed_dim, self.num_heads, self.num_kv_heads, self.head_dim = embed_dim, num_heads, num_kv_heads, head_dim
        self.max_seq_len, self.is_causal = max_seq_len, is_causal
        self.q_proj, self.k_proj, self.v_proj, self.output_proj = q_proj, k_proj, v_proj, output_proj
        self.pos_embeddings = pos_embeddings


class FeedForward(_WeightsOnly):
    """SwiGLU: w2(silu(w1 x) * w3 x); w1 = gate, w2 = down, w3 = up."""

    def __init__(self, gate_proj, down_proj, up_proj):
        super().__init__()
        self.w1, self.w2, self.w3 = gate_proj, down_proj, up_proj


class TransformerSelfAttentionLayer(_WeightsOnly):
    def __init__(self, attn, mlp, sa_norm, mlp_norm):
        super().__init__()
        self.attn, self.mlp, self.sa_norm, self.mlp_norm = attn, mlp, sa_norm, mlp_norm
        self.sa_scale, self.mlp_scale = nn.Identity(), nn.Identity()


class FourierEncoder(_WeightsOnly):
    """model.py:24-36: ``frequencies`` [1, F] ~ N(0, 1), ``proj`` Linear(2F -> E)."""

    def __init__(self, embed_dim, num_frequencies=128):
        super().__init__()
        self.frequencies = nn.Parameter(torch.randn(1, num_frequencies))
        self.proj = nn.Linear(2 * num_frequencies, embed_dim)


# ---------------------------------------------------------------------------
# Linear on the tcgen05 GEMM (the heads)
# ---------------------------------------------------------------------------
class Linear(nn.Linear):
    """``nn.Linear`` (same parameters, init and state dict) whose forward is
    the bf16 tcgen05 GEMM with an fp32 output (the ``cdk::linear`` op)."""

    def forward(self, x):
        if not x.is_cuda:
            _cuda_only("Linear")
        return torch.ops.cdk.linear(x, self.weight, self.bias)


class ValueHead(nn.Module):
    """model.py:39-52: Linear(E -> hidden) - Mish - Linear(hidden -> n_buckets)."""

    def __init__(self, embed_dim, n_buckets=100, hidden_size=256):
        super().__init__()
        self.mlp = nn.Sequential(Linear(embed_dim, hidden_size), nn.Mish(), Linear(hidden_size, n_buckets))

    def forward(self, hidden_state):
        return self.mlp(hidden_state)


# ---------------------------------------------------------------------------
# The backbone as one autograd node
# ---------------------------------------------------------------------------
class _Inputs:
    """The token-level inputs of one forward, in the engine's DeviceBatch field names."""
    __slots__ = ("ids", "wl_t", "d_t", "wl_pos", "d_pos", "slot", "frows")


class _Core:
    """Flat parameter store bound to a ChessDecoder's Parameter objects."""

    def __init__(self, model: "ChessDecoder", device: torch.device):
        self.cfg = model.cfg
        self.device = device
        self.store = ParamStore(self.cfg, device, optimizer_state=False)
        self.names = self.store.names()
        self.params = [model.get_parameter(n) for n in self.names]
        with torch.no_grad():
            for n, p in zip(self.names, self.params):
                if p.dtype != torch.float32:
                    raise TypeError(f"chessdecoder_b200.ChessDecoder keeps fp32 master weights; {n} is {p.dtype}")
                view = self.store.param(n)
                view.copy_(p.data)
                p.data = view
        self.backbone_idx = [i for i, n in enumerate(self.names) if not n.startswith(_HEADS)]
        self.ptrs = tuple(p.data_ptr() for p in self.params)
        self.versions = None
        self.backbone = Backbone(self.store, self.cfg)
        self.front = FrontEnd(self.store, self.cfg)

    def bound(self) -> bool:
        """False once a parameter was moved or replaced (``.to()``, assignment)."""
        return tuple(p.data_ptr() for p in self.params) == self.ptrs

    def refresh(self):
        v = tuple(p._version for p in self.params)
        if v != self.versions:
            self.store.refresh_bf16()
            self.versions = v

    def backbone_params(self):
        return [self.params[i] for i in self.backbone_idx]

    def grad_buffer(self):
        """The flat gradient buffer, as a 1-D fp32 tensor over its whole
        storage, if every backbone ``p.grad`` is the view of it that a backward
        of this core handed out (same storage, store offsets); else None."""
        st = self.store
        storage = None
        for i in self.backbone_idx:
            g = self.params[i].grad
            if g is None or g.dtype != torch.float32 or not g.is_contiguous():
                return None
            if storage is None:
                storage = g.untyped_storage()
                if storage.nbytes() != st.numel * 4:
                    return None
            elif g.untyped_storage().data_ptr() != storage.data_ptr():
                return None
            if g.storage_offset() != st.offsets[self.names[i]][0]:
                return None
        if storage is None:
            return None
        flat = torch.empty(0, dtype=torch.float32, device=self.device)
        flat.set_(storage, 0, (st.numel,), (1,))
        return flat

    def flat_grad_of(self, model=None):
        """The [first, last) range of the flat gradient buffer that holds the
        backbone gradients (None unless ``grad_buffer`` finds it)."""
        flat = self.grad_buffer()
        if flat is None:
            return None
        offs = [self.store.offsets[self.names[i]] for i in self.backbone_idx]
        lo = min(o for o, _, _ in offs)
        hi = max(o + n for o, _, n in offs)
        return flat[lo:hi]

    def plain_leaves(self) -> bool:
        """True when no backbone parameter carries gradient hooks, so the
        backward may write ``p.grad`` itself (see ops._bb_bwd)."""
        for i in self.backbone_idx:
            p = self.params[i]
            if p._backward_hooks or getattr(p, "_post_accumulate_grad_hooks", None):
                return False
        return True

    def inputs(self, x, wl_values, d_values, wl_positions, d_positions) -> _Inputs:
        B, S = x.shape
        dev = x.device
        t = _Inputs()
        t.ids = x.reshape(-1).to(torch.int64).contiguous()
        zf = None

        def vals(v):
            nonlocal zf
            if v is None:
                if zf is None:
                    zf = torch.zeros(B * S, device=dev)
                return zf
            return v.reshape(-1).to(torch.float32).contiguous()

        def pos(p):
            if p is None:
                return torch.zeros(B * S, device=dev, dtype=torch.uint8)
            return p.reshape(-1).to(torch.uint8).contiguous()

        t.wl_t, t.d_t = vals(wl_values), vals(d_values)
        t.wl_pos, t.d_pos = pos(wl_positions), pos(d_positions)
        # placeholder rows (one host sync, as the boolean indexing of model.py:177-180)
        t.frows = torch.nonzero(t.wl_pos | t.d_pos).reshape(-1).to(torch.int32)
        t.slot = torch.full((B * S,), -1, device=dev, dtype=torch.int32)
        t.slot[t.frows.long()] = torch.arange(t.frows.numel(), device=dev, dtype=torch.int32)
        return t


# ---------------------------------------------------------------------------
# ChessDecoder
# ---------------------------------------------------------------------------
class ChessDecoder(nn.Module):
    """model.py:55-194 on B200 kernels (same constructor, attributes, state
    dict and initial weights under the same ``torch.manual_seed``)."""

    def __init__(self, vocab_size, embed_dim=768, num_heads=12, num_layers=12, max_seq_len=2048, d_ff=None,
                 n_buckets=100, value_hidden_size=256, num_fourier_freq=128, wl_sigma=0.4):
        super().__init__()
        head_dim = embed_dim // num_heads
        d_ff = d_ff if d_ff is not None else 4 * embed_dim
        self.cfg = ModelConfig(vocab_size=vocab_size, embed_dim=embed_dim, num_heads=num_heads,
                               num_layers=num_layers, max_seq_len=max_seq_len, d_ff=d_ff, n_buckets=n_buckets,
                               value_hidden_size=value_hidden_size, num_fourier_freq=num_fourier_freq,
                               wl_sigma=wl_sigma)
        # construction order = the reference's, so the random draws match
        self.tok_embedding = nn.Embedding(vocab_size, embed_dim)
        rope = RotaryPositionalEmbeddings(dim=head_dim, max_seq_len=max_seq_len)
        self.layers = nn.ModuleList()
        for _ in range(num_layers):
            attn = MultiHeadAttention(
                embed_dim=embed_dim, num_heads=num_heads, num_kv_heads=num_heads, head_dim=head_dim,
                q_proj=nn.Linear(embed_dim, embed_dim, bias=False), k_proj=nn.Linear(embed_dim, embed_dim, bias=False),
                v_proj=nn.Linear(embed_dim, embed_dim, bias=False),
                output_proj=nn.Linear(embed_dim, embed_dim, bias=False), pos_embeddings=rope,
                max_seq_len=max_seq_len, is_causal=True)
            mlp = FeedForward(gate_proj=nn.Linear(embed_dim, d_ff, bias=False),
                              down_proj=nn.Linear(d_ff, embed_dim, bias=False),
                              up_proj=nn.Linear(embed_dim, d_ff, bias=False))
            self.layers.append(TransformerSelfAttentionLayer(attn=attn, mlp=mlp, sa_norm=RMSNorm(dim=embed_dim),
                                                             mlp_norm=RMSNorm(dim=embed_dim)))
        self.norm = RMSNorm(dim=embed_dim)
        self.board_head = Linear(embed_dim, V.board_vocab_size)
        self.policy_head = Linear(embed_dim, V.move_vocab_size)
        self.thinking_policy_head = Linear(embed_dim, V.move_vocab_size)
        self.wl_head = ValueHead(embed_dim, n_buckets, value_hidden_size)
        self.d_head = ValueHead(embed_dim, n_buckets, value_hidden_size)
        self.fourier_encoder = FourierEncoder(embed_dim, num_fourier_freq)
        self.register_buffer("wl_bucket_centers", make_wl_buckets(n_buckets, wl_sigma))
        self.register_buffer("d_bucket_centers", make_d_buckets(n_buckets))
        self._core: Optional[_Core] = None
        self._op_id = _ops.register_model(self)

    # -- flat parameter binding ------------------------------------------------
    @staticmethod
    def _is_backbone(name: str) -> bool:
        return not name.startswith(_HEADS)

    def _backbone_params(self):
        """The backbone Parameters in the flat store's order (what the
        ``cdk::backbone_fwd`` op receives), without binding the store."""
        if self._core is not None and self._core.bound():
            return self._core.backbone_params()
        from .engine import param_specs
        return [self.get_parameter(n) for n, _ in param_specs(self.cfg) if not n.startswith(_HEADS)]

    def _bind(self, device) -> _Core:
        core = self._core
        if core is None or core.device != device or not core.bound():
            core = self._core = _Core(self, device)
        core.refresh()
        return core

    @property
    def _store(self):
        """The flat parameter store (None before the first CUDA forward)."""
        return None if self._core is None else self._core.store

    def forward(self, x, input_pos=None, mask_type="causal", block_id=None, wl_values=None, d_values=None,
                wl_positions=None, d_positions=None):
        """x [B, S] token ids -> h [B, S, E] fp32 (final RMSNorm output), model.py:143-187.

        mask_type "causal" or "prefix" (causal + bidirectional inside each
        block_id run); the Fourier encoding of ``wl_values`` / ``d_values``
        replaces the embedding at ``wl_positions`` / ``d_positions`` (d wins
        where both are set).  ``input_pos`` ([S], or [B, S] with every row the
        same) gives the RoPE position of each sequence position (model.py:
        156-157); positions that differ between the sequences of a batch
        raise NotImplementedError.  The backbone is the ``cdk::backbone_fwd``
        op (chessdecoder_b200/ops.py)."""
        bsz, seq_len = x.shape
        prefix = mask_type != "causal"
        if prefix and block_id is None:
            raise ValueError("block_id is required for prefix mask mode")
        if not x.is_cuda:
            _cuda_only("ChessDecoder.forward")
        if seq_len > self.cfg.max_seq_len:
            raise ValueError(f"sequence length {seq_len} exceeds max_seq_len {self.cfg.max_seq_len}")
        pos = input_pos.reshape(-1, seq_len) if input_pos is not None else None
        h, _ = torch.ops.cdk.backbone_fwd(x, wl_values, d_values, wl_positions, d_positions,
                                          block_id if prefix else None, pos, self._op_id, self._backbone_params())
        return h

    def discretize_to_bucket(self, values, bucket_centers):
        """Nearest bucket centre (model.py:189-194; first index on ties)."""
        diffs = (values.unsqueeze(-1) - bucket_centers.unsqueeze(0)).abs()
        return bucket_centers[diffs.argmin(dim=-1)]


def soft_bucket_loss(logits, target_values, bucket_centers, valid_mask):
    """utils/training.py:24-50 on the soft two-bucket CE kernel: valid-masked
    mean of -sum(soft * log_softmax(logits)); a constant 0 (no graph) when
    there are no rows or no valid rows."""
    N = target_values.shape[0]
    traced = torch.compiler.is_compiling() or torch._guards.detect_fake_mode(logits) is not None
    if not traced and (N == 0 or valid_mask.sum() == 0):
        return torch.tensor(0.0, device=logits.device)
    if not logits.is_cuda:
        _cuda_only("soft_bucket_loss")
    return torch.ops.cdk.soft_bucket_ce(logits, target_values, bucket_centers, valid_mask)[0]


def prepare_fourier_inputs(model, wl_targets, d_targets, wl_positions, d_positions):
    """utils/training.py:114-133: zero tensors holding, at the WL / D
    placeholder positions, the targets snapped to the nearest bucket centre."""
    wl_in = torch.zeros_like(wl_targets)
    d_in = torch.zeros_like(d_targets)
    if wl_positions.any():
        wl_in[wl_positions] = model.discretize_to_bucket(wl_targets[wl_positions], model.wl_bucket_centers)
    if d_positions.any():
        d_in[d_positions] = model.discretize_to_bucket(d_targets[d_positions], model.d_bucket_centers)
    return wl_in, d_in


__all__ = ["ChessDecoder", "Linear", "ValueHead", "FourierEncoder", "RMSNorm", "soft_bucket_loss",
           "prepare_fourier_inputs"]
