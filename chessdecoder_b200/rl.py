"""GRPO policy-gradient step on the CUDA kernels: the compute path of
chessdecoder/rl (log_probs.py:19-190, grpo.py:58-126).

The reference runs the prefix pass of the model, gathers per-token log-probs
of the thinking head at ``thinking_move_mask`` rows and of the policy head at
``final_move_mask`` rows, and minimises the per-token clipped ratio objective
with a Schulman KL penalty, normalised by the number of action tokens.  Here:

* ``RLBatch`` / ``prepare_rl_batch``: the rollout batch on the device (token
  ids, block ids, Fourier placeholders, the action rows of each head with
  their targets, and per action row the rollout and reference log-probs and
  the sequence's advantage);
* ``GRPOStep.log_probs``: the prefix forward and the per-token log-probs
  (frozen / rollout policy; ``compute_ref_log_probs``);
* ``GRPOStep.forward_backward``: prefix forward, the two move heads on their
  action rows with the fused per-token GRPO kernel (``cdk_grpo_token``: log-
  softmax, ratio, clipping, KL, loss and the logit gradient in one pass), the
  backward through the backbone, gradients into the flat store;
  ``optimizer_step``: clip + AdamW as in training.

WL / D bucket actions (``wl_action_mask`` / ``d_action_mask``: only with the
reference's ``value_action_space=True``, off by default in
chessdecoder/rl/config.py, and recorded only by its C++ rollout engine) are
not built.
"""
from __future__ import annotations

import dataclasses
from typing import Optional

import numpy as np
import torch

from . import kernels as K
from . import vocab as V
from .engine import ModelConfig, TrainStep


@dataclasses.dataclass
class RLBatch:
    B: int
    S: int
    ids: torch.Tensor      # int64 [B*S]
    wl_t: torch.Tensor     # f32 [B*S] WL values (snapped to bucket centres in the Fourier kernel)
    d_t: torch.Tensor
    wl_pos: torch.Tensor   # u8 [B*S]
    d_pos: torch.Tensor
    slot: torch.Tensor     # i32 [B*S]
    frows: torch.Tensor    # i32 [Nf]
    bid: torch.Tensor      # i32 [B, S]
    heads: list            # [(head name, rows i32 [n], targets i32 [n], flat positions i64 [n], seq i64 [n])]
    old: Optional[list] = None   # per head: f32 [n] rollout log-probs
    ref: Optional[list] = None   # per head: f32 [n] reference log-probs
    adv: Optional[list] = None   # per head: f32 [n] advantages of the rows' sequences
    norm: Optional[torch.Tensor] = None  # f32 [1] = 1 / action tokens


def prepare_rl_batch(batch: dict, device, old_log_probs=None, ref_log_probs=None, advantages=None) -> RLBatch:
    """batch: the reference's rollout keys (``input_ids``, ``block_id``,
    ``wl_positions``, ``d_positions``, ``wl_values``, ``d_values``,
    ``thinking_move_mask``, ``final_move_mask``, ``move_token_ids``), all
    [B, S].  old / ref log-probs [B, S] and advantages [B] (any device) for the
    loss; without them only the log-probs can be computed."""
    dev = torch.device(device)
    ids = batch["input_ids"].cpu().numpy()
    Bn, S = ids.shape
    wl_pos = batch["wl_positions"].cpu().numpy().reshape(-1)
    d_pos = batch["d_positions"].cpu().numpy().reshape(-1)
    frows = np.nonzero(wl_pos | d_pos)[0].astype(np.int32)
    slot = np.full(Bn * S, -1, dtype=np.int32)
    slot[frows] = np.arange(frows.size, dtype=np.int32)
    tgt_all = batch["move_token_ids"].cpu().numpy().reshape(-1)
    heads = []
    n_act = 0
    for name, key in (("thinking_policy_head", "thinking_move_mask"), ("policy_head", "final_move_mask")):
        flat = np.nonzero(batch[key].cpu().numpy().reshape(-1))[0]
        n_act += flat.size
        heads.append((name, torch.from_numpy(flat.astype(np.int32)).to(dev),
                      torch.from_numpy(tgt_all[flat].astype(np.int32)).to(dev),
                      torch.from_numpy(flat.astype(np.int64)).to(dev),
                      torch.from_numpy((flat // S).astype(np.int64)).to(dev)))
    rb = RLBatch(B=Bn, S=S, ids=torch.from_numpy(ids.reshape(-1).astype(np.int64)).to(dev),
                 wl_t=batch["wl_values"].reshape(-1).float().to(dev), d_t=batch["d_values"].reshape(-1).float().to(dev),
                 wl_pos=torch.from_numpy(wl_pos.astype(np.uint8)).to(dev),
                 d_pos=torch.from_numpy(d_pos.astype(np.uint8)).to(dev), slot=torch.from_numpy(slot).to(dev),
                 frows=torch.from_numpy(frows).to(dev),
                 bid=batch["block_id"].to(torch.int32).to(dev).contiguous(), heads=heads)
    if old_log_probs is not None:
        old = old_log_probs.float().to(dev).reshape(-1)
        ref = ref_log_probs.float().to(dev).reshape(-1)
        adv = advantages.float().to(dev).reshape(-1)
        rb.old = [old.index_select(0, h[3]).contiguous() for h in heads]
        rb.ref = [ref.index_select(0, h[3]).contiguous() for h in heads]
        rb.adv = [adv.index_select(0, h[4]).contiguous() for h in heads]
        rb.norm = torch.tensor([1.0 / max(n_act, 1)], device=dev)
    return rb


class GRPOStep:
    """GRPO optimisation step of ChessDecoder on the CUDA kernels (the thinking
    head is trained, so the parameter store includes it)."""

    def __init__(self, cfg: ModelConfig, device="cuda", state_dict=None, lr=1e-6, weight_decay=0.1,
                 clip_epsilon_low=0.2, clip_epsilon_high=0.28, kl_coeff=0.05, max_norm=1.0, seed=0):
        """Defaults: chessdecoder/rl/config.py (lr 1e-6, wd 0.1, clip 0.2 / 0.28,
        KL 0.05, grad-norm clip 1.0; value actions off as ``value_action_space``)."""
        if not cfg.finetune:
            cfg = dataclasses.replace(cfg, finetune=True)
        self.cfg = cfg
        self.step_obj = TrainStep(cfg, device=device, seed=seed, lr=lr, weight_decay=weight_decay,
                                  max_norm=max_norm, state_dict=state_dict)
        self.store = self.step_obj.store
        self.device = self.step_obj.device
        self.eps_low, self.eps_high, self.kl_coeff = clip_epsilon_low, clip_epsilon_high, kl_coeff

    def _forward(self, rb: RLBatch):
        st = self.step_obj
        meta = K.attn_meta(rb.bid, rb.S)
        h0, fctx = st.front.forward(rb, n_copies=1)
        hN16, _, bctx = st.backbone.forward(h0, rb.B, 0, rb.S, rb.bid, meta)
        return hN16, fctx, bctx

    def _head(self, name, rows, tgt, hN16, old=None, ref=None, adv=None, norm=None, dhN=None, loss=None):
        st, E = self.store, self.cfg.embed_dim
        n = rows.numel()
        lp = torch.empty(n, device=self.device)
        if n == 0:
            return lp
        hp = torch.empty(n, E, device=self.device, dtype=torch.bfloat16)
        K.gather_rows_bf16(hN16, rows, hp)
        logits = torch.empty(n, V.move_vocab_size, device=self.device)
        K.gemm(hp, st.bf16(f"{name}.weight"), kind=K.EPI_STORE_F32, out=logits, bias=st.param(f"{name}.bias"))
        if old is None:
            K.grpo_token(logits, tgt, lp)
            return lp
        dl = torch.empty(n, 1928, device=self.device, dtype=torch.bfloat16)
        K.grpo_token(logits, tgt, lp, old, ref, adv, norm, self.eps_low, self.eps_high, self.kl_coeff, dlogits=dl,
                     dbias=st.grad_of(f"{name}.bias"), loss_out=loss, ncls=V.move_vocab_size)
        dhp = torch.empty(n, E, device=self.device)
        K.gemm(dl, st.bf16(f"{name}.weight"), b_mn=True, kind=K.EPI_STORE_F32, out=dhp, K=V.move_vocab_size)
        K.scatter_add_rows(dhp, rows, dhN)
        K.gemm(dl, hp, a_mn=True, b_mn=True, kind=K.EPI_ATOMIC_F32, out=st.grad_of(f"{name}.weight"),
               M=V.move_vocab_size, K=n)
        return lp

    def _scatter(self, rb: RLBatch, lps):
        out = torch.zeros(rb.B * rb.S, device=self.device)
        mask = torch.zeros(rb.B * rb.S, device=self.device, dtype=torch.bool)
        for (_, _, _, flat, _), lp in zip(rb.heads, lps):
            out.index_copy_(0, flat, lp)
            mask[flat] = True
        return out.view(rb.B, rb.S), mask.view(rb.B, rb.S)

    @torch.no_grad()
    def log_probs(self, rb: RLBatch):
        """Per-token log-probs [B, S] at the action positions and the action mask
        (compute_ref_log_probs / the rollout policy's log-probs)."""
        hN16, _, _ = self._forward(rb)
        return self._scatter(rb, [self._head(h[0], h[1], h[2], hN16) for h in rb.heads])

    def forward_backward(self, rb: RLBatch):
        """GRPO loss (device [1]) with every gradient in the store (zeroed
        here); also returns the current per-token log-probs [B, S]."""
        if rb.old is None:
            raise ValueError("the GRPO loss needs old / ref log-probs and advantages (prepare_rl_batch)")
        st = self.store
        st.grad.zero_()
        hN16, fctx, bctx = self._forward(rb)
        T, E = hN16.shape
        dhN = torch.zeros(T, E, device=self.device)
        loss = torch.zeros(1, device=self.device)
        lps = [self._head(h[0], h[1], h[2], hN16, rb.old[i], rb.ref[i], rb.adv[i], rb.norm, dhN, loss)
               for i, h in enumerate(rb.heads)]
        dh0 = self.step_obj.backbone.backward(dhN, bctx)
        self.step_obj.front.backward(rb, dh0, fctx, n_copies=1)
        return loss, self._scatter(rb, lps)[0]

    def optimizer_step(self):
        self.step_obj.optimizer_step()
