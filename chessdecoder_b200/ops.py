"""``torch.library`` custom ops ``cdk::*``: the drop-in module's compute as
operators with fake (meta) implementations and autograd formulas, so that
``loss.backward()`` (also through ``GradScaler``, chessdecoder/train/train.py:
245), FakeTensorMode shape propagation and ``torch.compile`` (graph breaks
around nothing: every op has a fake impl) see ordinary operators.

* ``cdk::linear(x, weight, bias) -> y`` and ``cdk::linear_backward`` -- the
  heads' Linear layers (bf16 tcgen05 GEMM, fp32 output and gradients).
* ``cdk::soft_bucket_ce(logits, target, centers, valid) -> (loss, dlogits)`` --
  utils/training.py:24-50; the gradient of the logits comes out of the same
  kernel and is the saved tensor of the autograd formula.
* ``cdk::backbone_fwd(...) -> (h, handle)`` and ``cdk::backbone_bwd_(handle,
  dh, grad)`` -- embedding + Fourier injection, every layer and the final
  norm (model.py:143-187).  The forward keeps its activations on the device
  for the backward; ``handle`` (a CPU int64 scalar) names them, and they are
  released when the handle is (normally: with the autograd graph).  The
  backward accumulates every backbone parameter's gradient into one flat fp32
  buffer (the engine's parameter layout), which is the op's declared mutated
  argument.
"""
from __future__ import annotations

import itertools
import weakref
from typing import List, Optional

import torch
from torch import Tensor

from . import kernels as K

# ---------------------------------------------------------------------------
# Linear (the heads)
# ---------------------------------------------------------------------------


def _pad(n: int, mult: int) -> int:
    return (n + mult - 1) // mult * mult


@torch.library.custom_op("cdk::linear", mutates_args=())
def linear(x: Tensor, weight: Tensor, bias: Optional[Tensor]) -> Tensor:
    """y = x W^T + b: bf16 operands, fp32 accumulation and output."""
    n_out, n_in = weight.shape
    if n_in % 8:
        raise ValueError("cdk::linear needs in_features % 8 == 0")
    x2 = x.reshape(-1, n_in)
    M = x2.shape[0]
    out = torch.empty(M, _pad(n_out, 4), device=x.device)
    if M:
        K.gemm(x2.to(torch.bfloat16).contiguous(), weight.detach().to(torch.bfloat16).contiguous(),
               kind=K.EPI_STORE_F32, out=out, bias=None if bias is None else bias.detach().contiguous(), N=n_out)
    return out[:, :n_out].reshape(*x.shape[:-1], n_out).clone()


@linear.register_fake
def _(x, weight, bias):
    return x.new_empty(*x.shape[:-1], weight.shape[0], dtype=torch.float32)


@torch.library.custom_op("cdk::linear_backward", mutates_args=())
def linear_backward(dy: Tensor, x: Tensor, weight: Tensor) -> List[Tensor]:
    """[dx, dW, db] of y = x W^T + b (dx fp32 in x's shape, dW, db fp32)."""
    n_out, n_in = weight.shape
    dy2 = dy.reshape(-1, n_out)
    M = dy2.shape[0]
    dy16 = torch.zeros(M, _pad(n_out, 8), device=dy.device, dtype=torch.bfloat16)
    dy16[:, :n_out] = dy2
    dx = torch.empty(M, n_in, device=dy.device)
    dw = torch.zeros(n_out, n_in, device=dy.device)
    if M:
        K.gemm(dy16, weight.detach().to(torch.bfloat16).contiguous(), b_mn=True, kind=K.EPI_STORE_F32, out=dx,
               K=n_out)
        K.gemm(dy16, x.reshape(-1, n_in).to(torch.bfloat16).contiguous(), a_mn=True, b_mn=True,
               kind=K.EPI_ATOMIC_F32, out=dw, M=n_out, K=M)
    else:
        dx.zero_()
    return [dx.reshape(x.shape), dw, dy2.float().sum(0)]


@linear_backward.register_fake
def _(dy, x, weight):
    n_out, n_in = weight.shape
    return [x.new_empty(x.shape, dtype=torch.float32), weight.new_empty(n_out, n_in, dtype=torch.float32),
            weight.new_empty(n_out, dtype=torch.float32)]


def _linear_setup(ctx, inputs, output):
    x, weight, bias = inputs
    ctx.save_for_backward(x, weight)
    ctx.has_bias = bias is not None


def _linear_bwd(ctx, dy):
    x, weight = ctx.saved_tensors
    dx, dw, db = torch.ops.cdk.linear_backward(dy, x, weight)
    return (dx.to(x.dtype) if ctx.needs_input_grad[0] else None, dw if ctx.needs_input_grad[1] else None,
            db if ctx.has_bias and ctx.needs_input_grad[2] else None)


linear.register_autograd(_linear_bwd, setup_context=_linear_setup)

# ---------------------------------------------------------------------------
# soft_bucket_loss
# ---------------------------------------------------------------------------


@torch.library.custom_op("cdk::soft_bucket_ce", mutates_args=())
def soft_bucket_ce(logits: Tensor, target: Tensor, centers: Tensor, valid: Tensor) -> List[Tensor]:
    """[loss (0-d), dlogits]: valid-masked mean over rows of -sum(soft *
    log_softmax(logits)) with two-bucket soft labels (utils/training.py:24-50)."""
    lg = logits.detach().to(torch.float32).contiguous()
    vf = valid.to(torch.float32).contiguous()
    norm = 1.0 / (vf.sum() + 1e-8)
    loss = torch.zeros(1, device=lg.device)
    dl = torch.empty_like(lg)
    K.soft_bucket_ce(lg, target.to(torch.float32).contiguous(), vf, centers.to(torch.float32).contiguous(),
                     norm.reshape(1), 1.0, dlogits=dl, loss_out=loss)
    return [loss.reshape(()), dl]


@soft_bucket_ce.register_fake
def _(logits, target, centers, valid):
    return [logits.new_empty((), dtype=torch.float32), logits.new_empty(logits.shape, dtype=torch.float32)]


def _sb_setup(ctx, inputs, output):
    ctx.save_for_backward(output[1])
    ctx.dtype = inputs[0].dtype


def _sb_bwd(ctx, grads):
    (dl,) = ctx.saved_tensors
    return (dl * grads[0]).to(ctx.dtype), None, None, None


soft_bucket_ce.register_autograd(_sb_bwd, setup_context=_sb_setup)

# ---------------------------------------------------------------------------
# Backbone
# ---------------------------------------------------------------------------
_MODELS: "weakref.WeakValueDictionary[int, object]" = weakref.WeakValueDictionary()
_SAVED: dict = {}
_IDS = itertools.count(1)


def register_model(model) -> int:
    """A process-wide id for a ChessDecoder, by which the ops find its flat
    parameter store (custom ops take tensors and scalars only)."""
    mid = next(_IDS)
    _MODELS[mid] = model
    return mid


def saved_count() -> int:
    """Backbone forwards whose activations are still held for a backward."""
    return len(_SAVED)


@torch.library.custom_op("cdk::backbone_fwd", mutates_args=())
def backbone_fwd(x: Tensor, wl_values: Optional[Tensor], d_values: Optional[Tensor],
                 wl_positions: Optional[Tensor], d_positions: Optional[Tensor], block_id: Optional[Tensor],
                 input_pos: Optional[Tensor], model_id: int, params: List[Tensor]) -> List[Tensor]:
    """[h (fp32 [B, S, E]), handle (CPU int64 scalar)]; prefix mask when
    block_id is given, causal otherwise; ``input_pos`` ([S] or [B, S] with
    equal rows) the RoPE position of each sequence position (None: 0..S-1).  ``params`` are the module's
    backbone Parameters (in the flat store's order), passed so that autograd
    connects their gradients; the kernels read the flat store they are bound
    to."""
    model = _MODELS[model_id]
    B, S = x.shape
    core = model._bind(x.device)
    inputs = core.inputs(x, wl_values, d_values, wl_positions, d_positions)
    prefix = block_id is not None
    bid32 = block_id.to(torch.int32).contiguous() if prefix else None
    h0, fctx = core.front.forward(inputs, n_copies=1, snap=False)
    meta = K.attn_meta(bid32, S) if prefix else None
    rope = None
    if input_pos is not None:
        pos = input_pos.reshape(-1, S)
        if pos.shape[0] > 1 and not bool((pos == pos[:1]).all()):
            raise NotImplementedError("cdk::backbone_fwd: input_pos must be the same for every sequence of the batch")
        pos = pos[0].to(device=x.device, dtype=torch.int64)
        if bool(((pos < 0) | (pos >= core.cfg.max_seq_len)).any()):
            raise ValueError(f"input_pos outside [0, max_seq_len={core.cfg.max_seq_len})")
        if not bool((pos == torch.arange(S, device=x.device)).all()):
            rope = core.backbone.rope[pos].contiguous()
    _, h32, bctx = core.backbone.forward(h0, B, 0 if prefix else B, S, bid32, meta, want_f32=True, rope=rope)
    key = next(_IDS)
    _SAVED[key] = (core, inputs, fctx, bctx)
    handle = torch.tensor(key, dtype=torch.int64)
    weakref.finalize(handle, _SAVED.pop, key, None)
    return [h32.view(B, S, core.cfg.embed_dim), handle]


@backbone_fwd.register_fake
def _(x, wl_values, d_values, wl_positions, d_positions, block_id, input_pos, model_id, params):
    B, S = x.shape
    E = _MODELS[model_id].cfg.embed_dim
    return [x.new_empty(B, S, E, dtype=torch.float32), torch.empty((), dtype=torch.int64, device="cpu")]


@torch.library.custom_op("cdk::backbone_bwd_", mutates_args=("grad",))
def backbone_bwd_(handle: Tensor, dh: Tensor, grad: Tensor) -> None:
    """Accumulates (+=) the gradient of every backbone parameter for the
    forward named by ``handle`` into ``grad`` (flat fp32, the parameter store's
    layout) and releases that forward's activations."""
    key = int(handle)
    if key not in _SAVED:
        raise RuntimeError("cdk::backbone_bwd_: the forward's activations were already released "
                           "(a second backward through the same graph needs retain_graph, which is not supported)")
    core, inputs, fctx, bctx = _SAVED.pop(key)
    st = core.store
    st.grad = grad
    try:
        dh0 = core.backbone.backward(dh.reshape(-1, core.cfg.embed_dim).to(torch.float32).contiguous(), bctx)
        core.front.backward(inputs, dh0, fctx, n_copies=1)
    finally:
        st.grad = None


@backbone_bwd_.register_fake
def _(handle, dh, grad):
    return None


def _bb_setup(ctx, inputs, output):
    ctx.handle = output[1]
    ctx.model_id = inputs[7]
    ctx.n_params = len(inputs[8])


def _bb_bwd(ctx, grads):
    """Eager: the backward writes straight into the flat buffer that backs
    every backbone ``p.grad`` (allocating it, and making its views the
    ``.grad``, on the first backward after ``zero_grad(set_to_none=True)``),
    so ``average_gradients`` reduces a few large slices in place.  Under
    tracing, or with gradient hooks on a parameter, the gradients are returned
    as views of a fresh buffer and autograd accumulates them."""
    dh = grads[0]
    model = _MODELS[ctx.model_id]
    tracing = torch.compiler.is_compiling() or torch._guards.detect_fake_mode(dh) is not None
    if tracing:
        from .engine import flat_layout
        offsets, numel = flat_layout(model.cfg)
        buf = dh.new_zeros(numel, dtype=torch.float32)
        torch.ops.cdk.backbone_bwd_(ctx.handle, dh, buf)
        views = [buf[o:o + n].view(shape) for name, (o, shape, n) in offsets.items() if model._is_backbone(name)]
        return (None,) * 8 + (views,)
    core = model._core
    st = core.store
    direct = core.plain_leaves() and not torch.is_grad_enabled()
    buf = core.grad_buffer() if direct else None
    fresh = buf is None
    if fresh:
        buf = dh.new_zeros(st.numel, dtype=torch.float32)
    torch.ops.cdk.backbone_bwd_(ctx.handle, dh, buf)
    views = [st._view(buf, core.names[i]) for i in core.backbone_idx]
    head = (None,) * 8
    if not direct:
        return head + (views,)
    if fresh:
        for i, g in zip(core.backbone_idx, views):
            p = core.params[i]
            if p.grad is None:
                p.grad = g
            else:
                p.grad.add_(g)
    return head + ([None] * ctx.n_params,)


backbone_fwd.register_autograd(_bb_bwd, setup_context=_bb_setup)
